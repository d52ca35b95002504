// Prompt-pass convolution: a thread owns one channel and slides its window
// down 16 rows, forming every B*x product once; the history update runs
// after all windows read the old history.
#include "common.cuh"
#include "conv.cuh"
#include "kernels.cuh"

namespace lfm3 {
namespace {

constexpr int kConvRows = 16;
constexpr int kMaxWidth = 32;

__device__ __forceinline__ float product(const float* p, const float* history,
                                         int source, int ch, int H, int L) {
  return source >= 0 ? p[size_t(source) * 3 * H + ch] *
                           p[size_t(source) * 3 * H + 2 * H + ch]
                     : history[size_t(ch) * (L - 1) + (L - 1) + source];
}

// kL > 0: the width as a compile-time constant (window and taps stay in
// registers); kL == 0: any width L <= kMaxWidth.
template <int kL>
__global__ void conv_window_kernel(const float* __restrict__ p,
                                   const float* __restrict__ w,
                                   const float* __restrict__ history,
                                   float* __restrict__ y, int n, int H,
                                   int L_runtime) {
  constexpr int kCap = kL > 0 ? kL : kMaxWidth;
  const int L = kL > 0 ? kL : L_runtime;
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  const int first = blockIdx.y * kConvRows;
  if (ch >= H)
    return;
  float taps[kCap], window[kCap];
#pragma unroll
  for (int t = 0; t < kCap; ++t)
    if (t < L)
      taps[t] = w[size_t(ch) * L + t];
  grid_dependency_wait();
  allow_dependents();
#pragma unroll
  for (int t = 0; t < kCap - 1; ++t)
    if (t < L - 1)
      window[t + 1] = product(p, history, first - (L - 1) + t, ch, H, L);
  const int last = min(first + kConvRows, n);
  for (int row = first; row < last; ++row) {
#pragma unroll
    for (int t = 0; t < kCap - 1; ++t)
      if (t < L - 1)
        window[t] = window[t + 1];
    window[L - 1] = product(p, history, row, ch, H, L);
    float sum = 0;
#pragma unroll
    for (int t = 0; t < kCap; ++t)
      if (t < L)
        sum = fmaf(taps[t], window[t], sum);
    y[size_t(row) * H + ch] = sum * p[size_t(row) * 3 * H + H + ch];
  }
}

__global__ void conv_history_kernel(const float* __restrict__ p,
                                    float* history, int n, int H, int L) {
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= H)
    return;
  grid_dependency_wait();
  allow_dependents();
  float past[kMaxWidth];
  for (int j = 0; j < L - 1; ++j)
    past[j] = product(p, history, n - (L - 1) + j, ch, H, L);
  for (int j = 0; j < L - 1; ++j)
    history[size_t(ch) * (L - 1) + j] = past[j];
}

}  // namespace

cudaError_t launch_short_conv(const float* p, const float* w, float* history,
                              float* y, int n, int H, int L, bool update,
                              cudaStream_t stream, bool pdl) {
  if (L < 2 || L > kMaxWidth || n < 0)
    return cudaErrorInvalidValue;
  if (n == 0)
    return cudaSuccess;
  const dim3 grid((H + 127) / 128, (n + kConvRows - 1) / kConvRows);
  // the LFM3 width (l_cache) as a compile-time constant
  cudaError_t e = launch_kernel(L == 7 ? conv_window_kernel<7>
                                       : conv_window_kernel<0>,
                                grid, dim3(128), 0, stream, pdl, p, w,
                                static_cast<const float*>(history), y, n, H, L);
  if (e != cudaSuccess || !update)
    return e;
  return launch_kernel(conv_history_kernel, dim3((H + 127) / 128), dim3(128), 0,
                       stream, pdl, p, history, n, H, L);
}

}  // namespace lfm3
