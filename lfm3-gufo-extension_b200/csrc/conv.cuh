// Gated short convolution of prompt rows (the decode step's convolution is
// fused into the in_proj projection epilogue, q8_gemv.cu).
#pragma once
#include <cuda_runtime.h>

namespace lfm3 {

// p = [B | C | x] rows of in_proj (FP32, 3H per row), w = f32 [H][L],
// history = the last L - 1 B*x products before the first row (channel-major,
// f32 [H][L - 1]). y[t][ch] = (sum_j w[ch][j] * bx[t - L + 1 + j]) * C[t][ch],
// FMA chain oldest first. With update, history becomes the last L - 1
// products (ConvolutionWindow / ConvolutionHistory / ConvolutionStep,
// hip/ops.hip:971-1044, 1135-1151).
cudaError_t launch_short_conv(const float* p, const float* w, float* history,
                              float* y, int n, int H, int L, bool update,
                              cudaStream_t stream, bool pdl = false);

}  // namespace lfm3
