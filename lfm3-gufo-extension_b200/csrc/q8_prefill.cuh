// Q8_0 projections of prompt rows (16..512 per pass) with FP16 row-scaled
// activations: y[t][m] = scale[t] * sum_b d[m][b] * (sum_{k in b} q[m][k] *
// x16[t][k]), FP32 accumulation per K32 block (hip/q8_prefill.hpp:94-645,
// RegQ8Gemm / TiledQ8Gemm, and LaunchSplit, hip/ops.hip:2039-2119).
#pragma once
#include <cuda.h>
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
  // TMA maps: weights as [rows][row_bytes / 16][16] with boxes of 272-byte
  // chunks (128 rows for Plain, 64 rows for SwiGLU gate and up), and the
  // activations as [rows of the buffer][K] fp16 with 128 x 32 boxes,
  // 64-byte swizzle.
  alignas(64) CUtensorMap w_maps[4];
  alignas(64) CUtensorMap x_map;
  int kind;
  int K;
  int tokens;
  int x_row0;   // first activation row of this pass in x_map
  int n_out;
  PrefillOutput o[4];
  int first_tile[5];  // row tiles (128 rows) of each output
  int row_tiles;
  const float* scale;   // [tokens]
  unsigned* row_max;    // SwiGLU: FP32 bits of each row's max |out|
};

// Fills p.w_maps and p.x_map (x is [x_rows][K] fp16; the pass reads rows
// x_row0 .. x_row0 + tokens - 1) and launches.
cudaError_t launch_q8_prefill(PrefillParams p, const __half* x, int x_rows,
                              cudaStream_t stream);

}  // namespace lfm3
