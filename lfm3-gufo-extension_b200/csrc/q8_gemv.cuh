// Q8_0 projections of up to eight FP32 rows (the decode step's GEMV / skinny
// GEMM). Replaces SmallBatchQ8_0ExactFp32VecGEMMKernel, Q8_0GEMV and
// Q8_0MultiGEMV (hip/ops.hip:304-406, 671-856) and the SwiGLU and
// convolution-step kernels that follow them (hip/ops.hip:165-182,
// 1135-1151).
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "decode_types.cuh"

namespace lfm3 {

constexpr int kGemvRows = 64;     // weight rows per tile
constexpr int kGemvBlocks = 8;    // Q8 blocks per stage (256 columns)
constexpr int kGemvChunk = kGemvBlocks * 34;  // bytes per row per stage
constexpr int kGemvStages = 4;
constexpr int kGemvWarps = 8;     // consumer warps, one Q8 block each
constexpr int kGemvThreads = (kGemvWarps + 1) * 32;
constexpr int kGemvTile = kGemvRows * kMaxBatch;  // fp32 values per tile

enum GemvKind : int {
  // out[token * ld + row] for up to four weights sharing the input
  kGemvPlain = 0,
  // tile = 32 gate rows + the same 32 up rows; writes silu(g) * u as split
  // activations of width F
  kGemvSwiGLU = 1,
  // tile = 16 channels: rows ch, H + ch, 2H + ch of in_proj (B, C, x);
  // runs the width-L convolution step against each row's session history
  // and writes the gated output as split activations of width H
  kGemvConv = 2,
};

struct GemvOutput {
  const uint8_t* w;  // Q8_0 rows of K / 32 blocks
  float* out;
  int rows;
  int ld;
};

struct GemvParams {
  // TMA maps over the weight rows (tensor_map.hpp), 272-byte chunks: Plain
  // one per output with 64-row boxes; SwiGLU gate and up with 32-row boxes;
  // Conv in_proj with 16-row boxes.
  alignas(64) CUtensorMap maps[4];
  int kind;
  int K;        // columns (multiple of 256)
  int chunks;   // K / 256
  int tiles;
  int tokens;   // 1..8
  int n_out;
  GemvOutput o[4];
  int first_tile[5];
  const void* x;      // split input, [tokens][K / 8] records
  void* split_out;    // SwiGLU / Conv output (split)
  int split_width;    // its row length
  // Conv epilogue
  const float* conv_w;    // f32 [H][L]
  const DecodeRows* rows;
  int layer;
  int H;
  int L;
  // stream-K fix-up scratch
  float* partials;    // [grid][2][kGemvTile]
  unsigned* tickets;  // [tiles], zero between launches
};

// Grid size and scratch needs of one launch.
int gemv_grid(int units, int sms);
size_t gemv_partial_floats(int grid);

// Box rows of the weight maps each kind reads (per output slot).
inline int gemv_box_rows(int kind) {
  return kind == kGemvPlain ? kGemvRows : kind == kGemvSwiGLU ? 32 : 16;
}
// Encodes p.maps from p.o[j].w / rows / K (host; for callers without a map
// cache).
cudaError_t fill_gemv_maps(GemvParams& p);

}  // namespace lfm3
