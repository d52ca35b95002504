// Q8_0 projections of prompt rows (16..512 per pass) with FP16 row-scaled
// activations: y[t][m] = scale[t] * sum_b d[m][b] * (sum_{k in b} q[m][k] *
// x16[t][k]), FP32 accumulation per K32 block (hip/q8_prefill.hpp:94-645,
// RegQ8Gemm / TiledQ8Gemm, and LaunchSplit, hip/ops.hip:2039-2119).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lfm3 {

enum PrefillKind : int {
  kPrefillPlain = 0,   // up to four weights sharing the input
  kPrefillSwiGLU = 1,  // o[0] gate, o[1] up: out = silu(g) * u, row maxima
};

struct PrefillOutput {
  const uint8_t* w;
  float* out;  // [tokens][ld]
  int rows;
  int ld;
};

struct PrefillParams {
  int kind;
  int K;
  int tokens;
  int n_out;
  PrefillOutput o[4];
  int first_tile[5];  // row tiles of each output
  int row_tiles;
  const __half* x;      // [tokens][K]
  const float* scale;   // [tokens]
  unsigned* row_max;    // SwiGLU: FP32 bits of each row's max |out|
};

cudaError_t launch_q8_prefill(PrefillParams p, cudaStream_t stream);

}  // namespace lfm3
