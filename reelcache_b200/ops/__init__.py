"""Python entry points of the sm_100a kernels (tcgen05 GEMM, fused restore, attention, norms, RoPE,
fitter reductions, quantize + mosaic). Each op raises when the native extension is missing on a CUDA
device: there is no silent eager fallback on the GPU path."""
