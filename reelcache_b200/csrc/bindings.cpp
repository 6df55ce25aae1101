// Python bindings of the reelcache_b200 native extension (CUDA kernels for sm_100a and the C++
// host fast paths).
#include <torch/extension.h>

#include <vector>

namespace rc {
void gemm_bf16_tn(const at::Tensor& A, const at::Tensor& B, at::Tensor& out, int64_t epilogue,
                  const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& gate,
                  const c10::optional<at::Tensor>& resid, double alpha, int64_t bn,
                  const c10::optional<at::Tensor>& status);
void restore_launch(const at::Tensor& jobs, const std::vector<at::Tensor>& a_ops, const std::vector<at::Tensor>& b_ops,
                    const at::Tensor& inverse, const c10::optional<at::Tensor>& status);
void prep_launch(const at::Tensor& jobs, int64_t device);
void colminmax(const at::Tensor& p, at::Tensor& lo, at::Tensor& hi, at::Tensor& bad);
void quantize_columns(const at::Tensor& p, const at::Tensor& scale, const at::Tensor& offset, at::Tensor& out);
void rope_store_launch(const at::Tensor& jobs);
void unpack_launch(const at::Tensor& jobs, int64_t device);
}  // namespace rc

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "reelcache_b200 native kernels (sm_100a) and host fast paths";
  m.def("gemm_bf16_tn", &rc::gemm_bf16_tn, "out = epilogue(alpha * A @ B^T) on tcgen05", py::arg("A"),
        py::arg("B"), py::arg("out"), py::arg("epilogue") = 0, py::arg("bias") = py::none(),
        py::arg("gate") = py::none(), py::arg("resid") = py::none(), py::arg("alpha") = 1.0, py::arg("bn") = 0,
        py::arg("status") = py::none());
  m.def("restore_launch", &rc::restore_launch, "fused restore GEMM over <= 16 jobs", py::arg("jobs"),
        py::arg("a_ops"), py::arg("b_ops"), py::arg("inverse"), py::arg("status") = py::none());
  m.def("colminmax", &rc::colminmax, "per-column extrema of FP32 coefficients", py::arg("p"), py::arg("lo"),
        py::arg("hi"), py::arg("bad"));
  m.def("quantize_columns", &rc::quantize_columns, "FP64 rint quantization of coefficients to uint8",
        py::arg("p"), py::arg("scale"), py::arg("offset"), py::arg("out"));
  m.def("prep_launch", &rc::prep_launch, "scaled hi/lo basis + bias preparation over <= 48 jobs", py::arg("jobs"),
        py::arg("device"));
  m.def("rope_store_launch", &rc::rope_store_launch, "dense RoPE + cast + strided store over <= 48 jobs",
        py::arg("jobs"));
  m.def("unpack_launch", &rc::unpack_launch, "mosaic pictures -> dense uint8 [N, K_pad] over <= 48 jobs",
        py::arg("jobs"), py::arg("device"));
}
