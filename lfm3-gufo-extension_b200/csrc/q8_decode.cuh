// Decode projections over a fragment-ordered copy of the Q8_0 weights.
//
// The decode round reads every Q8_0 matrix once per round for <= 8 rows, so
// it is bound by HBM bandwidth only if the per-weight instruction stream is
// short. The GGUF layout (34-byte blocks {fp16 d; int8 qs[32]}) makes every
// thread shift bytes into place before it can convert them, so at load time
// the engine repacks each matrix the round reads (Model::Load) into records
// of one 16-row m-tile x one 32-column block:
//
//   bytes   0..511  codes q + 128 (u8) in mma.sync m16n8k16 A-fragment
//                   order: lane l = 4g + c holds row g's columns 8c..8c+7,
//                   then row g + 8's (16 bytes, one 128-bit load)
//   bytes 512..543  half2 {d(row g), d(row g + 8)} for g = 0..7
//
// 544 bytes per 512 weights, the GGUF size, so a round moves the same bytes.
// BF16 matrices (the numerical-reference weights) get the same layout with
// 1024-byte records: lane l = 4g + c holds row g's columns 8c..8c+7 at
// bytes 16 l and row g + 8's at 512 + 16 l, the values themselves.
// Records are ordered [tile][block][m-tile of the tile], so a unit of work
// (one tile x 16 or 32 blocks) is one contiguous run of memory that a single
// bulk copy brings into shared memory.
//
// Replaces the reference's SmallBatchQ8_0ExactFp32VecGEMMKernel, Q8_0GEMV,
// Q8_0MultiGEMV (hip/ops.hip:304-406, 671-856) and the SwiGLU and
// convolution-step kernels that follow them (hip/ops.hip:165-182,
// 1135-1151) on the engine's decode path.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "decode_types.cuh"

namespace lfm3 {

constexpr int kDecRecord = 544;  // bytes per (m-tile, block) record, Q8_0
constexpr int kDecRecordBf16 = 1024;  // the same for BF16 matrices
constexpr int kDecWarps = 8;     // consumer warps
constexpr int kDecThreads = (kDecWarps + 1) * 32;  // + the producer warp
// Shared-memory ring: 9 slots of 17 KB units, 6 of 26 KB, 4 of 35 KB.
constexpr int kDecRingBytes = 156672;
constexpr int kDecMaxSlots = 9;
// Projections with K <= kDecStagedK keep the round's input records in
// shared memory (bulk copies of unit-sized column chunks per token, each
// chunk on its own barrier; rows padded by 16 bytes so the fragment loads
// hit distinct banks) beside a smaller ring: 8 slots of 17 KB, 5 of 26 KB,
// 4 of 35 KB.
constexpr int kDecStagedK = 2048;
constexpr int kDecMaxXChunks = kDecStagedK / (32 * 8);  // units of >= 8 blocks
constexpr int kDecXRowBytes = kDecStagedK * 4 + 16;
constexpr int kDecRingStaged = 139264;
constexpr int kDecMaxMtiles = 4;

enum DecodeKind : int {
  // up to four outputs sharing the input; m-tiles of the outputs in order
  kDecPlain = 0,
  // tile = kMT / 2 m-tiles of gate rows then the same rows of up; writes
  // silu(gate) * up
  kDecSwiGLU = 1,
  // tile = 16 channels: their B, C and x rows of in_proj; runs the
  // convolution step against each row's session history
  kDecConv = 2,
};

// Which source rows a packed group holds (host and device).
struct DecodeLayout {
  int kind;
  int mt;     // m-tiles per tile: Plain 1, 2 or 4; SwiGLU 2 or 4; Conv 3
  int K;      // columns, a multiple of 512
  int tiles;
  int n_src;  // Plain: outputs (1..4); SwiGLU 2 (gate, up); Conv 1 (in_proj)
  // Plain: first m-tile of each output in the concatenation, [n_src] = all
  int first_mtile[5];
  int rows[4];  // rows of each source matrix
  int H;        // Conv: channels (in_proj has 3H rows)
  int bf16;     // BF16 matrices (1024-byte records) instead of Q8_0
  // Plain sources that are column ranges of wider matrices (a K split):
  // source j's rows are src_ld[j] bytes apart (0: K / 32 x 34, or 2 K for
  // BF16) and read the input columns x_col[j] .. x_col[j] + K - 1 of input
  // rows x_ld wide (0: K). No tile may span two such sources.
  int src_ld[4];
  int x_col[4];
  int x_ld;
};

// Source matrix j and first row of m-tile m of tile t; false for padding.
__host__ __device__ inline bool decode_mtile_source(const DecodeLayout& l,
                                                    int t, int m, int& j,
                                                    int& row0) {
  if (l.kind == kDecPlain) {
    const int gm = t * l.mt + m;
    if (gm >= l.first_mtile[l.n_src])
      return false;
    j = 0;
    for (int q = 1; q < l.n_src; ++q)
      if (gm >= l.first_mtile[q])
        j = q;
    row0 = (gm - l.first_mtile[j]) * 16;
    return true;
  }
  const int half = l.kind == kDecSwiGLU ? l.mt / 2 : l.mt / 3;
  const int part = m / half;  // SwiGLU: gate / up; Conv: B / C / x
  const int sub = m % half;
  if (l.kind == kDecSwiGLU) {
    j = part;
    row0 = (t * half + sub) * 16;
    return true;
  }
  j = 0;
  row0 = part * l.H + (t * half + sub) * 16;
  return true;
}

// Completes a layout from kind, K, n_src, rows[] (and H for Conv): picks the
// m-tiles per tile so that the busiest of `sms` CTAs holds as few m-tiles as
// possible, fills first_mtile and tiles. False for unsupported shapes.
bool decode_layout(DecodeLayout& l, int sms);
// Bytes of the packed copy.
size_t decode_packed_bytes(const DecodeLayout& l);
// Packs the GGUF Q8_0 rows of src[j] (device memory, K / 32 x 34 bytes per
// row) into dst (decode_packed_bytes, 16-byte aligned).
cudaError_t launch_decode_pack(const DecodeLayout& l,
                               const uint8_t* const src[4], uint8_t* dst,
                               cudaStream_t stream);

struct DecodeOut {
  float* out;  // FP32 [token][ld]
  int ld;
};

struct DecodeParams {
  DecodeLayout layout;
  const uint8_t* w;  // the packed copy
  int tokens;        // 1..8
  const void* x;     // split input records [tokens][K / 8] (common.cuh),
                     // 16-byte aligned
  DecodeOut o[4];    // Plain outputs
  void* split_out;   // SwiGLU / Conv: split records [tokens][split_width]
  int split_width;
  float* f32_out;  // SwiGLU: optional FP32 copy [token][f32_ld]
  int f32_ld;
  // Conv
  const float* conv_w;  // f32 [H][L]
  const DecodeRows* rows;
  int layer;
  int L;
  // Optional: the first prefetch_bytes of the next projection's packed copy,
  // asked into L2 in equal slices by the CTAs once their own weight copies
  // are issued, so the next launch's CTAs (resident only after these leave)
  // read their first units from L2 rather than HBM. 16-byte aligned.
  const uint8_t* prefetch;
  size_t prefetch_bytes;
};

// CTAs of a launch: one per SM, at most one per tile.
int decode_grid(const DecodeLayout& l, int sms);
cudaError_t launch_decode_gemv(const DecodeParams& p, int grid,
                               cudaStream_t stream, bool pdl);

}  // namespace lfm3
