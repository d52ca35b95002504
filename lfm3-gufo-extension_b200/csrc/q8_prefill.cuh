// Q8_0 projections of prompt rows (16..512 per pass) with FP16 row-scaled
// activations: y[t][m] = scale[t] * sum_b d[m][b] * (sum_{k in b} q[m][k] *
// x16[t][k]), FP32 accumulation (hip/q8_prefill.hpp:94-645, RegQ8Gemm /
// TiledQ8Gemm, and LaunchSplit, hip/ops.hip:2039-2119).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace lfm3 {

enum PrefillKind : int {
  kPrefillPlain = 0,   // up to four weights sharing the input
  kPrefillSwiGLU = 1,  // o[0] gate, o[1] up: out = silu(g) * u, row maxima
};

// A work tile is 256 weight rows (two tensor-memory accumulators of 128)
// by 256 prompt rows; SwiGLU tiles pair 128 gate rows with the same 128 up
// rows.
constexpr int kPrefillTileRows = 256;
constexpr int kPrefillTileTokens = 256;
// Split-K: at most this many (tile, K range) units keep FP32 partial sums
// (hip/ops.hpp:17-21, kMaxSplitUnits).
constexpr int kPrefillMaxSplitUnits = 128;
constexpr size_t kPrefillPartialFloats =
    size_t(kPrefillMaxSplitUnits) * kPrefillTileRows * kPrefillTileTokens;

struct PrefillOutput {
  const uint8_t* w;
  float* out;  // [tokens][ld]
  int rows;
  int ld;
};

struct PrefillParams {
  // TMA maps (filled by launch_q8_prefill): weights as [rows][row_bytes / 8]
  // 8-byte elements with boxes of 34 elements (8 blocks) x 256 rows (128
  // for SwiGLU gate and up), and the activations as [rows of the buffer][K]
  // fp16 with 256 x 32 boxes, 64-byte swizzle.
  alignas(64) CUtensorMap w_maps[4];
  alignas(64) CUtensorMap x_map;
  int kind;
  int K;
  int tokens;
  int x_row0;   // first activation row of this pass in x_map
  int n_out;
  PrefillOutput o[4];
  // filled by launch_q8_prefill
  int first_tile[5];  // 256-row tiles of each output (Plain)
  int row_tiles;
  int splits;         // K ranges per tile
  const float* scale;   // [tokens]
  unsigned* row_max;    // SwiGLU: FP32 bits of each row's max |out|
  // Optional split-K workspace of kPrefillPartialFloats floats (16-byte
  // aligned); without it no projection splits K.
  float* partial;
  // Plain with one output only: a projection that splits K leaves its FP32
  // partial sums in `partial` ([row tile][token tile][split] blocks of
  // [256 prompt rows][256 output rows], row scales not applied) for the
  // consumer to add in split order, instead of reducing them into o[0].out
  bool keep_splits;
  // BF16 weights (the numerical-reference models) instead of Q8_0: the
  // weight tiles come straight from [rows][K] bf16 by TMA, and x is three
  // bf16 planes (split_bf16_rows) whose sum is the FP32 input exactly,
  // plane q's rows at q * x_rows of the buffer; scale may be null (1).
  int bf16;
  int x_plane_rows;  // filled by launch_q8_prefill: x_rows
};

// Fills the maps and the tiling of p (x is [x_rows][K] fp16, or for bf16
// [3][x_rows][K] bf16 planes; the pass reads rows x_row0 .. x_row0 +
// tokens - 1) and launches. K must be a multiple of 256.
// *splits (optional) receives the K ranges used: with keep_splits set and
// more than one, the output is left as partial sums in `partial`.
cudaError_t launch_q8_prefill(PrefillParams p, const void* x, int x_rows,
                              cudaStream_t stream, int* splits = nullptr,
                              bool pdl = false);

}  // namespace lfm3
