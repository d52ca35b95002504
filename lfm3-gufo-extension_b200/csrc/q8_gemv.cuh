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

enum GemvKind : int {
  // out[token * ld + row] for up to four weights sharing the input;
  // tile = 16 rows of one weight (64 for tall projections), chunks of 32 Q8
  // blocks (1024 columns) or 16
  kGemvPlain = 0,
  // tile = 16 gate rows + the same 16 up rows, chunks of 32 blocks; writes
  // silu(g) * u as split activations of width F (and/or FP32)
  kGemvSwiGLU = 1,
  // tile = 16 channels: rows ch, H + ch, 2H + ch of in_proj (B, C, x),
  // chunks of 16 blocks; runs the width-L convolution step against each
  // row's session history and writes the gated output as split activations
  kGemvConv = 2,
};

// m-tiles (16 rows each) of a tile: Plain 1, or 4 for projections with at
// least two 64-row tiles per CTA slot (the input fragments of a block then
// serve four m-tiles); SwiGLU 2; Conv 3. The 16-byte units a row occupies in
// shared memory for chunks of `blocks` Q8 blocks (the chunk plus padding
// that spreads the rows of a warp's fragment loads over the banks).
constexpr __host__ __device__ int gemv_mtiles(int kind, int wide = 0) {
  return kind == kGemvPlain ? (wide ? 4 : 1) : kind == kGemvSwiGLU ? 2 : 3;
}
constexpr __host__ __device__ int gemv_pitch_units(int blocks) {
  return blocks * 34 / 16 + ((blocks * 34 / 16) % 4 == 0 ? 2 : 0);
}

// The weight ring: kGemvRingBytes split into as many equal slots (<= 8) as
// one chunk of the kernel's kind fits, so several chunks stay in flight.
constexpr int kGemvRingBytes = 73728;
constexpr int kGemvMaxSlots = 8;
constexpr int kGemvWarps = 8;  // consumer warps
constexpr int kGemvThreads = (kGemvWarps + 1) * 32;

struct GemvOutput {
  const uint8_t* w;  // Q8_0 rows of K / 32 blocks
  float* out;
  int rows;
  int ld;
};

struct GemvParams {
  // TMA maps over the weight rows (encode_q8_rows, tensor_map.hpp): boxes of
  // gemv_box_rows(p) rows x gemv_pitch_units(chunk_blocks) * 16 bytes: Plain
  // one per output, SwiGLU gate and up, Conv in_proj.
  alignas(64) CUtensorMap maps[4];
  int kind;
  int K;             // columns
  int chunk_blocks;  // Q8 blocks per chunk (64, 32 or 16; gemv_plan)
  int chunks;        // K / (32 * chunk_blocks)
  int wide;          // Plain: 64-row tiles (chunks of 16 blocks)
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
};

// Fills p.chunk_blocks, p.chunks, p.wide, p.tiles and p.first_tile from the
// kind, K, outputs and the SM count (Plain: 64-row tiles in chunks of 16
// blocks when there are at least two per CTA slot, else 16-row tiles in
// chunks of 32 blocks when K allows, else 16; SwiGLU 32 or 16; Conv 16);
// returns false for widths that are not multiples of 512.
bool gemv_plan(GemvParams& p, int sms);
// Rows of one TMA box (16 x m-tiles of a Plain tile, 16 otherwise).
int gemv_box_rows(const GemvParams& p);
int gemv_grid(int tiles, int sms);
// Encodes p.maps from p.o[j].w / rows / K (host; for callers without a map
// cache).
cudaError_t fill_gemv_maps(GemvParams& p);

// ---- BF16 projections ----------------------------------------------------------
// Exact BF16 x FP32 on the CUDA cores with FP32 accumulation, for the BF16
// numerical-reference weights (Wave32GEMVKernel_1Row, FastGEMVBlockKernel,
// BatchedExactBf16GEMMFp32VecKernel, hip/ops.hip:184-302, 452-591,
// 1917-2005). Same GemvParams as the Q8_0 kernel (o[j].w are BF16 rows of K
// elements; maps unused) with tiles of 16 x m-tiles rows: Plain 16, SwiGLU
// 16 gate + 16 up, Conv 16 channels x (B, C, x).
//   x32 == nullptr: decode rows, p.x split records of p.tokens <= 8 rows
//     (hi + lo, 22 significant bits of each FP32 input), and the kind's
//     epilogue exactly as q8_gemv_kernel's;
//   otherwise FP32 prompt rows x32[t * x_ld + k], t < rows, in groups of 8:
//     Plain, or SwiGLU writing FP32 silu(g) * u to o[0].out.
// K must be a multiple of 256.
bool bf16_plan(GemvParams& p);
cudaError_t launch_bf16_gemv(const GemvParams& p, const float* x32, int x_ld,
                             int rows, cudaStream_t stream);

}  // namespace lfm3
