/* CPU oracle for the LFM3 backbone step — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's FP32 scalar oracle
 * (reference.cpp:9-168, Reference::Step). Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may load it, and only as the checker or the
 * timed CPU baseline; the product path never calls it.
 *
 * Parity pin: tests compare this restatement bit for bit against the
 * reference's own reference.cpp/weights.cpp/config.cpp compiled unmodified
 * into oracle/_ref (see oracle/Makefile) and against golden vectors that
 * compiled reference produced (tests/golden/).
 */
#ifndef LFM3_ORACLE_H_
#define LFM3_ORACLE_H_
#include "../include/lfm3_types.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct lfm3_oracle lfm3_oracle;

/* Reference::Reference (reference.cpp:45-63). threads > 1 splits each
 * matrix-vector product by rows; every row keeps the reference's summation
 * order, so results do not depend on the thread count. NULL on invalid
 * context or allocation failure. */
lfm3_oracle* lfm3_oracle_create(const lfm3_weights* weights, uint32_t context,
                                int threads);
void lfm3_oracle_destroy(lfm3_oracle* oracle);
/* Reference::Reset (reference.cpp:64-71). */
void lfm3_oracle_reset(lfm3_oracle* oracle);
/* Reference::Step (reference.cpp:72-168). logits may be NULL (no head).
 * Returns 0, or -1 for an invalid token or a full context. */
int lfm3_oracle_step(lfm3_oracle* oracle, uint32_t token, float* logits);
uint32_t lfm3_oracle_position(const lfm3_oracle* oracle);
/* Test-only numerics switch (off by default, no counterpart in
 * reference.cpp): round every stored K and V value to the nearest fp16, as
 * the engine's F16 rings hold them (engine.cpp:71-72), where reference.cpp
 * keeps FP32 (reference.cpp:113-115). Isolates that one storage difference
 * in GPU-vs-oracle comparisons. */
void lfm3_oracle_set_kv_half(lfm3_oracle* oracle, int on);
/* The fp16 rounding that switch applies (round to nearest even, overflow
 * to infinity), for tests. */
float lfm3_oracle_round_half(float value);
/* Final hidden state after the last step's final norm (valid when that step
 * produced logits). */
const float* lfm3_oracle_hidden(const lfm3_oracle* oracle);

#ifdef __cplusplus
}
#endif
#endif
