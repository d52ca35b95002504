/* Deterministic synthetic LFM3 weights (no checkpoint is available).
 *
 * Every matrix element is an approximately normal value (Irwin-Hall sum of
 * four 16-bit uniforms from a counter-based splitmix64 hash of
 * (seed, tensor index, element index)), scaled to std 0.02 and rounded to
 * BF16. Q8_0 matrices quantise those BF16 values with the llama.cpp rule:
 * per 32 values d = amax / 127 (stored as fp16), q = roundf(x / d) computed
 * as roundf(x * (1 / d)) with the fp32 d. Norm weights are 1.0 (plus an
 * optional jitter for tests), RoPE factors are [1] * (D / 4) followed by
 * [1e30] * (D / 4), and the output projection is tied to the embedding
 * (weights.cpp:55-57). Tensor indices follow the binding order of
 * weights.cpp:54-93, so the same seed always yields the same model
 * regardless of thread count.
 */
#ifndef LFM3_SYNTH_H_
#define LFM3_SYNTH_H_
#include "lfm3_types.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lfm3_synth_model {
  lfm3_weights weights;
  void* storage; /* one host allocation holding every tensor payload */
  size_t storage_bytes;
} lfm3_synth_model;

/* The graded geometry: hidden 2048, FFN 8192, 16 Q / 4 KV heads of 128,
 * vocab 65536, window 256, conv width 7, context 262144, eps 1e-5,
 * theta 1e6 / 1e4, 24 layers in the order CCSGCCSGCCSGCCSGCCSGCCGC
 * (C conv, S sliding attention, G global attention). */
void lfm3_synth_default_config(lfm3_config* config);

/* Sets the layer order from a string of 'C', 'S' and 'G' (one per layer)
 * with kv_heads KV heads on attention layers. Returns 0, or -1 if the
 * string is empty, too long or holds another character. */
int lfm3_synth_set_layers(lfm3_config* config, const char* pattern,
                          uint32_t kv_heads);

/* Allocates and fills a model. matrix_type is LFM3_Q8_0 or LFM3_BF16.
 * norm_jitter adds norm_jitter * N(0,1)-like noise to every norm weight
 * (0 for the graded config). threads <= 0 uses every online core.
 * Returns 0 on success, or a negative code on invalid geometry or
 * allocation failure. */
int lfm3_synth_generate(const lfm3_config* config, uint64_t seed,
                        uint32_t matrix_type, float norm_jitter, int threads,
                        lfm3_synth_model* out);
void lfm3_synth_free(lfm3_synth_model* model);

/* Bytes of one row of a matrix of this type and width (0 if unsupported). */
size_t lfm3_row_bytes(uint32_t type, uint32_t cols);

/* Round-to-nearest-even conversions used by the generator and the tests. */
uint16_t lfm3_float_to_half(float value);
float lfm3_half_to_float(uint16_t bits);

#ifdef __cplusplus
}
#endif
#endif
