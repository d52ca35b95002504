// Gated GQA attention over the F16 K/V rings: the decode kernel (all rows of
// a round, ragged depths, one launch per layer) and the prompt kernels.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "decode_types.cuh"

namespace lfm3 {

constexpr int kHeadDim = 128;
constexpr int kDecodeTile = 64;     // keys per tile
constexpr int kMaxDecodeSplits = 64;

struct DecodeAttentionParams {
  const float* q;      // [rows][heads * 128]
  const float* k;      // [rows][kv_heads * 128]
  const float* v;
  const float* gate;   // [rows][heads]
  int ldq, ldk, ldg;   // row strides (floats)
  const float* q_norm;
  const float* k_norm;
  const float* freq;     // [64] frequencies of this layer's theta
  const float* factors;  // [64] or null (sliding layers)
  const DecodeRows* rows;
  int layer;
  int heads, kv_heads;
  int window;  // 0: full attention
  int max_splits;  // key spans per (row, KV group), <= kMaxDecodeSplits
  // > 0: key tiles per span instead (every row's spans about equally long,
  // as many spans as that takes, up to kMaxDecodeSplits)
  int span_tiles;
  // spans launched per (row, KV group): at least the most any row of the
  // round uses (decode_spans_used); 0 launches kMaxDecodeSplits
  int span_grid;
  // 1 when every ring row before a row's position was complete before the
  // launch's stream predecessor started (the engine launches a round's first
  // kernel only after all earlier work of the batch's streams): the kernel
  // then fetches its first key tile while that predecessor still runs
  int ring_settled;
  float eps;
  void* out_split;   // [rows][heads * 128] split records
  float* out_f32;    // optional [rows][heads * 128]
  float* partials;   // [rows][heads][kMaxDecodeSplits][130]
  unsigned* tickets; // [kMaxBatch][kv_heads], zero between launches
  // Operator form (rows == nullptr): one row at `position` whose q is
  // already normalised and rotated; key `position` comes from chunk_k /
  // chunk_v and earlier keys from the ring (the reference's Attention with
  // n == 1, hip/ops.hip:2289-2315).
  int position;
  const __half* ring_k;
  const __half* ring_v;
  const __half* chunk_k;
  const __half* chunk_v;
  int capacity;
};

// Per-head Q/K RMSNorm + RoPE, the F16 K/V store into each row's ring slot
// position % capacity, and attention over keys
// [max(0, position + 1 - window), position], all rows of a round in one
// launch (DecodeHeadsKernel + DecodeWaves + DecodeCombine,
// hip/ops.hip:1072-1134, 1562-1691, 1710-1728).
cudaError_t launch_decode_attention(const DecodeAttentionParams& p, int rows,
                                    cudaStream_t stream, bool pdl);

size_t decode_attention_partial_floats(int heads);
// Key tiles per span of a row with `tiles` key tiles.
__host__ __device__ inline int decode_span_tiles(int tiles, int max_splits,
                                                 int span_tiles) {
  const int fit = (tiles + kMaxDecodeSplits - 1) / kMaxDecodeSplits;
  if (span_tiles > 0)
    return span_tiles > fit ? span_tiles : fit;
  const int splits = max_splits < 1                  ? 1
                     : max_splits > kMaxDecodeSplits ? kMaxDecodeSplits
                                                     : max_splits;
  return (tiles + splits - 1) / splits;
}
// Key tiles of a row at `position` and the spans the decode attention kernel
// uses for it.
int decode_key_tiles(int position, int window);
int decode_spans_used(int position, int window, int max_splits,
                      int span_tiles);

// ---- prompt pass ------------------------------------------------------------

// Per-head Q/K RMSNorm + RoPE of n prompt rows starting at position, in
// place on q and k (FP32), and the F16 K/V rows written to k16/v16 rows
// 0..n-1 (hip/ops.hip:1072-1134 over rows, PromptHeads).
cudaError_t launch_prompt_heads(float* q, float* k, const float* v, int ldq,
                                int ldk, const float* q_norm,
                                const float* k_norm, const float* freq,
                                const float* factors, __half* k16, __half* v16,
                                int n, int heads, int kv_heads, int position,
                                float eps, cudaStream_t stream,
                                bool pdl = false);

// Causal attention of n prompt rows at position: keys at or after position
// from k16/v16 (chunk rows), earlier keys from the ring (slot t % capacity),
// window > 0 limits each query to its last `window` keys. FP16 Q (scaled by
// rsqrt(D) log2 e) and probabilities on the tensor cores, FP32 softmax and
// accumulation; output gated by 1 / (1 + exp(-gate)) (WmmaAttn +
// PromptCombine, hip/ops.hip:1355-1561, 1692-1709).
cudaError_t launch_prompt_attention(const float* q, int ldq, const __half* k16,
                                    const __half* v16, const __half* ring_k,
                                    const __half* ring_v, const float* gate,
                                    int ldg, float* out, int n, int heads,
                                    int kv_heads, int position, int capacity,
                                    int window, float* scratch,
                                    cudaStream_t stream, bool pdl = false);
size_t prompt_attention_scratch_floats(int heads, int rows, int keys);

// The same attention with window 0 when every key, the chunk's own
// included, is already in the ring (position + n <= capacity, no wrap): the
// prompt pass of the full-attention layers. tcgen05 tensor cores with
// TMA-loaded K/V tiles; the same FP16 roundings of Q and P, the same spans
// and the same scratch as launch_prompt_attention.
cudaError_t launch_prompt_attention_tc(const float* q, int ldq,
                                       const __half* ring_k,
                                       const __half* ring_v, const float* gate,
                                       int ldg, float* out, int n, int heads,
                                       int kv_heads, int position,
                                       int capacity, float* scratch,
                                       cudaStream_t stream, bool pdl = false);
// Merges the spans' (maximum, sum, output) partials of either kernel and
// applies the gate.
cudaError_t launch_prompt_combine(const float* partial, const float* gate,
                                  int ldg, float* out, int n, int heads,
                                  int spans, cudaStream_t stream,
                                  bool pdl = false);

// Copies the last min(n, capacity) chunk rows into the ring at
// position (hip/ops.hip:1737-1749).
cudaError_t launch_store_kv(const __half* k16, const __half* v16,
                            __half* ring_k, __half* ring_v, int n, int stride,
                            int position, int capacity, cudaStream_t stream,
                            bool pdl = false);

}  // namespace lfm3
