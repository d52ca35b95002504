/* Plain-C model description shared by the CUDA library, the host engine and
 * the CPU oracle.
 *
 * These structs restate the reference's host types as POD so they can cross
 * a C ABI:
 *   lfm3_config   <- gufo::models::lfm3::Config       (config.hpp:8-20)
 *   lfm3_tensor   <- gufo::models::lfm3::Tensor       (weights.hpp:7-12)
 *   lfm3_layer    <- gufo::models::lfm3::LayerWeights (weights.hpp:13-18)
 *   lfm3_weights  <- gufo::models::lfm3::Weights      (weights.hpp:19-26)
 * Tensor payloads keep the GGUF encodings byte for byte: F32, F16, BF16 rows
 * and Q8_0 rows of 34-byte blocks {fp16 d; int8 qs[32]}.
 */
#ifndef LFM3_TYPES_H_
#define LFM3_TYPES_H_
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GgmlType values used by the reference (gguf_reader.hpp GgmlType). */
enum lfm3_dtype {
  LFM3_F32 = 0,
  LFM3_F16 = 1,
  LFM3_Q8_0 = 8,
  LFM3_BF16 = 30,
};

/* LayerType (config.hpp:7). */
enum lfm3_layer_type {
  LFM3_CONV = 0,
  LFM3_FULL_ATTENTION = 1,
  LFM3_SLIDING_ATTENTION = 2,
};

#define LFM3_MAX_LAYERS 256
#define LFM3_Q8_BLOCK 32
#define LFM3_Q8_BLOCK_BYTES 34

typedef struct lfm3_config {
  uint32_t hidden, intermediate, vocab, context, heads, head_dim;
  uint32_t window, conv_width, n_layers;
  float eps, theta, theta_swa;
  uint32_t kv_heads[LFM3_MAX_LAYERS]; /* 0 for convolution layers */
  uint32_t layer_type[LFM3_MAX_LAYERS]; /* enum lfm3_layer_type */
} lfm3_config;

typedef struct lfm3_tensor {
  const void* data; /* NULL when absent */
  uint32_t type;    /* enum lfm3_dtype */
  uint32_t cols, rows;
  size_t bytes;
} lfm3_tensor;

typedef struct lfm3_layer {
  lfm3_tensor norm, ffn_norm, post_norm, post_ffn_norm;
  lfm3_tensor gate, up, down;
  lfm3_tensor conv, in_proj, out_proj;
  lfm3_tensor q, k, v, q_norm, k_norm, attn_gate, attn_out;
} lfm3_layer;

typedef struct lfm3_weights {
  lfm3_config config;
  lfm3_tensor embedding, output, output_norm, rope_freqs;
  lfm3_layer layers[LFM3_MAX_LAYERS];
} lfm3_weights;

#ifdef __cplusplus
}
#endif
#endif
