// Row kernels around the projections: token embedding, the fused
// residual-add + sandwich RMSNorm, and FP32 -> FP16 row-scaled conversion.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lfm3 {

// Where a normalised row goes. Any subset may be set.
struct NormOut {
  float* f32;      // [rows][H] FP32
  void* split;     // [rows][H / 8] split records (decode projections)
  __half* half;    // [rows][H] FP16 scaled by 2^e (prompt projections)
  float* scale;    // [rows] 2^-e for half
};

// A residual branch still split over K: the FP32 partial sums of a prompt
// projection, one [256 prompt rows][256 output rows] block per (tile, split)
// with tile = output row tile * token_tiles + prompt row tile; the branch
// is scale[prompt row] * (sum of the splits in split order); a null scale
// (BF16 projections) is 1.
constexpr int kSplitTileFloats = 256 * 256;
struct SplitBranch {
  const float* partial;
  const float* scale;
  int splits;
  int token_tiles;
  // with a plain branch: a second FP32 branch [rows][H] added after it (the
  // other half of a decode projection split over K)
  const float* second;
};

// x += RMSNorm_post(branch) (when branch, or split; post_w may be null:
// plain add), then out = RMSNorm(x) * norm_w (when norm_w).
// hip/ops.hip:890-970.
cudaError_t launch_residual_norm(const float* branch, const float* post_w,
                                 float* x, const float* norm_w, NormOut out,
                                 int rows, int H, float eps,
                                 cudaStream_t stream, bool pdl,
                                 const SplitBranch* split = nullptr,
                                 const float* branch2 = nullptr);

// x[r] = embedding row ids[r] (F32 / F16 / BF16 / Q8_0 rows), then out =
// RMSNorm(x) * norm_w. hip/ops.hip:858-875 fused with the first norm.
// ids == nullptr takes the token from the decode rows descriptor (tokens).
cudaError_t launch_embed_norm(const void* table, uint32_t type,
                              const uint32_t* ids, const uint32_t* tokens,
                              float* x, const float* norm_w, NormOut out,
                              int rows, int H, float eps, cudaStream_t stream,
                              bool pdl);

// FP32 rows -> FP16 scaled so each row's maximum magnitude lies in
// [2^14, 2^15), with scale 2^-e (hip/q8_prefill.hpp:27-51). With row_max
// (FP32 bits of each row's maximum, known already) the reduction is skipped
// (hip/q8_prefill.hpp:52-74).
cudaError_t launch_half_rows(const float* x, const unsigned* row_max,
                             __half* values, float* scale, int rows, int K,
                             cudaStream_t stream, bool pdl = false);

// FP32 rows -> three bf16 planes whose sum is each value exactly (plane q
// the round-to-nearest bf16 of what planes 0 .. q - 1 left): plane q of row
// r at planes + (q * plane_rows + r) * K elements. The BF16 prompt
// projections read them (K a multiple of 8, 16-byte aligned rows).
cudaError_t launch_split_bf16_rows(const float* x, void* planes, int rows,
                                   int K, int plane_rows, cudaStream_t stream,
                                   bool pdl = false);

// FP32 rows -> split records (x = hi + lo, fp16 each).
// Up to kMaxRowCopies FP32 row copies in one launch (16-byte pieces when
// both rows are 16-byte aligned and the length a multiple of 4): the end of
// a decode round hands each session its frontier and logits rows.
constexpr int kMaxRowCopies = 16;
struct RowCopies {
  const float* src[kMaxRowCopies];
  float* dst[kMaxRowCopies];
  int floats[kMaxRowCopies];
  int vector[kMaxRowCopies];  // set by launch_row_copies
  int count;
  // optional: receives the device error word once every earlier kernel in
  // the stream has finished (host-mapped memory)
  unsigned* error_out;
};
cudaError_t launch_row_copies(const RowCopies& c, cudaStream_t stream,
                              bool pdl);

cudaError_t launch_split_rows(const float* x, void* split, int rows, int K,
                              cudaStream_t stream);

}  // namespace lfm3
