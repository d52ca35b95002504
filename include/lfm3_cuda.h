/* C ABI of the B200 (sm_100a) LFM3 backbone step library, liblfm3_cuda.so.
 *
 * Two layers, both plain C: pointers, sizes, POD descriptors, no exceptions.
 *
 * 1. Operators (lfm3_cuda_*): one entry point per function of the
 *    reference's operator surface, namespace gufo::models::lfm3::gpu in
 *    hip/ops.hpp (cited per function). Pointer arguments are device
 *    pointers, `stream` is a cudaStream_t passed as void* (NULL: legacy
 *    default stream), tensors are lfm3_tensor descriptors whose data points
 *    to device memory in the reference's GGUF encodings.
 * 2. Engine (lfm3_model_* / lfm3_session_*): the reference's Model and
 *    Session (engine.hpp:17-163) over those operators. Host buffers unless
 *    stated.
 *
 * Every function returns LFM3_OK (0) or a negative LFM3_ERR_* code; the
 * message of the last failure on the calling thread is lfm3_last_error().
 * The reference's operators return void / bool and throw
 * std::invalid_argument on unsupported shapes (hip/ops.hip:2293-2294); here
 * those become LFM3_ERR_UNSUPPORTED and nothing is launched.
 */
#ifndef LFM3_CUDA_H_
#define LFM3_CUDA_H_
#include <stddef.h>
#include <stdint.h>

#include "lfm3_types.h"

#ifdef __cplusplus
extern "C" {
#endif

enum lfm3_status {
  LFM3_OK = 0,
  LFM3_ERR_INVALID = -1,     /* bad argument or refused input */
  LFM3_ERR_CUDA = -2,        /* a CUDA call failed */
  LFM3_ERR_UNSUPPORTED = -3, /* shape or format this build does not run */
  LFM3_ERR_POISONED = -4,    /* session needs lfm3_session_reset */
  LFM3_ERR_DEVICE_WAIT = -5, /* a bounded device wait gave up */
};

/* Message of the last failure on this thread ("" if none). */
const char* lfm3_last_error(void);
/* Reads and clears the device error word set by bounded waits that gave up
 * (0: none). */
unsigned lfm3_cuda_take_device_error(void);
/* Diagnostic with no counterpart in the reference (its kernels do not bound
 * their waits): one kernel whose wait nothing ends gives up after limit_us
 * (1..1000000) and leaves code 5 in the device error word; the context stays
 * usable. Exercises the failure path of every bounded wait. */
int lfm3_cuda_wait_probe(unsigned limit_us, void* stream);

/* ---- operators (hip/ops.hpp) -------------------------------------------- */

/* DenseWorkspace (hip/ops.hpp:21-26): quantized holds FP16 prompt
 * activations or split decode activations, row_max one word per row,
 * partial the FP32 split-K partial sums of prompt projections with few
 * tiles (added in split order by a reduce pass). tickets keeps the
 * reference's layout; this build's split-K needs no tickets and leaves it
 * untouched. */
typedef struct lfm3_dense_workspace {
  void* quantized;
  unsigned* row_max;
  float* partial;
  unsigned* tickets;
} lfm3_dense_workspace;

/* DenseWorkspaceBytes (hip/ops.hpp:27): bytes of `quantized` for rows x K. */
size_t lfm3_cuda_dense_workspace_bytes(size_t rows, size_t K);
/* Bytes of `partial` and words of `tickets` (SplitPartialBytes,
 * hip/ops.hpp:35; kMaxSplitUnits, hip/ops.hpp:28). */
size_t lfm3_cuda_split_partial_bytes(void);
size_t lfm3_cuda_split_ticket_words(void);
/* kPromptRows (hip/ops.hpp:33): projections of at least this many rows
 * read FP16 row-scaled activations; fewer rows keep FP32 inputs (as two
 * fp16 terms on the tensor cores). */
int lfm3_cuda_prompt_rows(void);

/* Embed (hip/ops.hpp:13-14): out[r] = row tokens[r] of weight, FP32. */
int lfm3_cuda_embed(const lfm3_tensor* weight, const uint32_t* tokens,
                    float* out, int n, void* stream);

/* Dense (hip/ops.hpp:72-73): out[n][rows] = x[n][cols] . weight^T. */
int lfm3_cuda_dense(const lfm3_tensor* weight, const float* x, float* out,
                    int n, void* stream, const lfm3_dense_workspace* workspace);

/* Output (hip/ops.hpp:37-40). */
typedef struct lfm3_output {
  const lfm3_tensor* weight;
  float* out;
} lfm3_output;

/* Project (hip/ops.hpp:46-48): up to four weights with the same column
 * count read one input. split_ready (hip/ops.hpp:44-45): the workspace
 * already holds this input as FP16 prompt activations (written by
 * lfm3_cuda_residual_norm with split set, for the same n rows and width), so
 * x is not read; it applies to Q8_0 prompt rows (n >= kPromptRows) and is
 * ignored otherwise. */
int lfm3_cuda_project(const lfm3_output* outputs, int count, const float* x,
                      int n, void* stream,
                      const lfm3_dense_workspace* workspace, int split_ready);
/* ProjectSwiGLU (hip/ops.hpp:51-53): out = silu(gate x) * (up x). */
int lfm3_cuda_project_swiglu(const lfm3_tensor* gate, const lfm3_tensor* up,
                             const float* x, float* out, float* up_scratch,
                             int n, void* stream,
                             const lfm3_dense_workspace* workspace,
                             int split_ready);
/* ProjectFfn (hip/ops.hpp:55-58): out = down(silu(gate x) * (up x)), the
 * activation left in hidden; split_ready applies to the gate/up input. */
int lfm3_cuda_project_ffn(const lfm3_tensor* gate, const lfm3_tensor* up,
                          const lfm3_tensor* down, const float* x,
                          float* hidden, float* up_scratch, float* out, int n,
                          void* stream, const lfm3_dense_workspace* workspace,
                          int split_ready);

/* ResidualNorm (hip/ops.hpp:62-65): x += post_norm(branch) (branch and
 * post_norm may be NULL), then z = norm(x) unless norm is NULL. With split
 * set, z goes to workspace->quantized as FP16 prompt activations instead.
 * Returns LFM3_ERR_UNSUPPORTED for widths this build does not run (the
 * reference returns false). */
int lfm3_cuda_residual_norm(const float* branch, const lfm3_tensor* post_norm,
                            float* x, const lfm3_tensor* norm, float* z, int n,
                            int hidden, float eps, int split, void* stream,
                            const lfm3_dense_workspace* workspace);

/* ShortConv (hip/ops.hpp:76-78): gated width-L causal convolution over n
 * rows of projection [B | C | x] (3 * hidden floats per row), reading
 * history (f32 [hidden][L - 1]) before the first row and, with update,
 * storing the last L - 1 B*x products back into it. */
int lfm3_cuda_short_conv(const float* projection, const float* weight,
                         float* history, float* out, int n, int hidden,
                         int width, void* stream, int update);

/* RopeFrequencies (hip/ops.hpp:80): out[i] = float(pow(double theta,
 * -2i/dim)), dim / 2 values. */
int lfm3_cuda_rope_frequencies(float* out, int dim, float theta, void* stream);
/* Rope (hip/ops.hpp:81-82): rotates pairs (i, i + dim/2) of n rows of heads
 * heads by (position + row) * frequencies[i] / factors[i] (factors may be
 * NULL). */
int lfm3_cuda_rope(float* x, const float* frequencies, const float* factors,
                   int n, int heads, int dim, int position, void* stream);

/* Attention (hip/ops.hpp:94-98): causal gated GQA attention of n query
 * rows at position. Keys at or after position come from k/v (n F16 rows),
 * earlier keys from the ring cache_k/cache_v (slot t % capacity); window > 0
 * keeps each query's last `window` keys. n == 1 keeps Q and probabilities
 * in FP32; prompts use FP16 Q and probabilities on the tensor cores. dim
 * must be 128 and heads / kv_heads 2, 4 or 8. */
int lfm3_cuda_attention(const float* q, const uint16_t* k, const uint16_t* v,
                        const float* gate, const uint16_t* cache_k,
                        const uint16_t* cache_v, float* out, int n, int heads,
                        int kv_heads, int dim, int position, int capacity,
                        int window, void* stream, float* scratch);
/* No counterpart in the reference. The n == 1 case of lfm3_cuda_attention
 * for callers that cannot allocate device memory (a serving loop whose
 * memory is a fixed arena sized at start-up, or a latency-critical thread
 * that must not call cudaMalloc between steps): same arguments minus n and
 * scratch; its scratch is a static device array of about 1 MiB per GPU that
 * loads the library, kept until the process exits, so heads must be <= 32
 * (LFM3_ERR_UNSUPPORTED with a message beyond that). It allocates nothing.
 * The first call on each device looks up that array's device address (and
 * again the first call after cudaDeviceReset, whose new context holds the
 * array afresh); make it before any stream capture. Calls share the array:
 * calls that overlap on the GPU race and must be serialised by the caller. */
int lfm3_cuda_attention_decode_noalloc(const float* q, const uint16_t* k,
                                       const uint16_t* v, const float* gate,
                                       const uint16_t* cache_k,
                                       const uint16_t* cache_v, float* out,
                                       int heads, int kv_heads, int dim,
                                       int position, int capacity, int window,
                                       void* stream);
/* No counterpart in the reference: lfm3_cuda_attention with window 0 when
 * every key, the chunk's own included, is already in the cache (store the
 * chunk with lfm3_cuda_store_kv first; position + n <= capacity, so nothing
 * wraps). The engine's prompt pass of the full-attention layers: tcgen05
 * tensor cores with TMA-loaded key tiles, the same FP16 roundings of Q and
 * probabilities and the same scratch as lfm3_cuda_attention. n >= 1. */
int lfm3_cuda_attention_stored(const float* q, const float* gate,
                               const uint16_t* cache_k,
                               const uint16_t* cache_v, float* out, int n,
                               int heads, int kv_heads, int dim, int position,
                               int capacity, void* stream, float* scratch);
/* AttentionScratchBytes (hip/ops.hpp:99). */
size_t lfm3_cuda_attention_scratch_bytes(int heads, int dim, int context,
                                         int rows);

/* PromptHeads / DecodeHeads (hip/ops.hpp:133-146): per-head Q/K RMSNorm
 * and RoPE in place on q and k; F16 K and V rows to k16/v16 rows 0..n-1
 * (prompt) or to ring slot position % capacity (decode). */
int lfm3_cuda_prompt_heads(float* q, float* k, const float* v,
                           const float* q_norm, const float* k_norm,
                           const float* frequencies, const float* factors,
                           uint16_t* k16, uint16_t* v16, int n, int heads,
                           int kv_heads, int dim, int position, float eps,
                           void* stream);
int lfm3_cuda_decode_heads(float* q, float* k, const float* v,
                           const float* q_norm, const float* k_norm,
                           const float* frequencies, const float* factors,
                           uint16_t* cache_k, uint16_t* cache_v, int heads,
                           int kv_heads, int dim, int position, int capacity,
                           float eps, void* stream);

/* StoreKV (hip/ops.hpp:126-127) and PackKV (hip/ops.hpp:123-124). */
int lfm3_cuda_store_kv(const uint16_t* k, const uint16_t* v, uint16_t* cache_k,
                       uint16_t* cache_v, int n, int stride, int position,
                       int capacity, void* stream);
int lfm3_cuda_pack_kv(const float* k, const float* v, uint16_t* k16,
                      uint16_t* v16, size_t count, void* stream);
/* SelectRows (hip/ops.hpp:120-121): copies packed rows rows[i] of source. */
int lfm3_cuda_select_rows(const lfm3_tensor* source, const uint32_t* rows,
                          void* out, int count, void* stream);

/* SharesSplit (hip/ops.hpp:41-43): 1 when these projections of n rows read
 * one FP16 prompt input (n >= kPromptRows, Q8_0 weights of one width and a
 * workspace to hold it), else 0. Host only. */
int lfm3_cuda_shares_split(const lfm3_output* outputs, int count, int n,
                           const lfm3_dense_workspace* workspace);
/* LaunchBatchedResidualAdd (hip/ops.hpp:156-158): out = a + b over batch x
 * dim floats (out may be a); dim a multiple of 8, at most 8192. */
int lfm3_cuda_batched_residual_add(const float* a, const float* b, float* out,
                                   size_t batch, size_t dim, void* stream);
/* LaunchGEMV (hip/ops.hpp:163-164), LaunchBatchedQuantGEMMFp32
 * (hip/ops.hpp:165-168) and LaunchExactBf16GEMMFp32SmallBatch
 * (hip/ops.hpp:169-171): y[r] = W x[r] for rows of FP32 x ([rows][K]) and a
 * [M][K] matrix (Q8_0 with K a multiple of 512, or BF16 with K a multiple
 * of 256), the results of lfm3_cuda_dense. They take no workspace: the Q8_0
 * input conversion uses stream-ordered memory (cudaMallocAsync /
 * cudaFreeAsync on `stream`). */
int lfm3_cuda_gemv(const void* A, uint32_t a_type, const float* x, float* y,
                   size_t M, size_t K, void* stream);
/* Decode projections over the fragment-ordered copy that the engine packs
 * its matrices into at load (no reference counterpart: the reference's
 * decode GEMVs read the GGUF rows directly; this exposes the engine's decode
 * kernel on caller-supplied matrices). w[0..n_w) are Q8_0 matrices, or BF16
 * matrices (all of one type), of K columns (K a multiple of 512); BF16
 * products use each input as three exact bf16 terms of its 22-bit split. swiglu == 0: n_w <= 4 outputs,
 * out[j][r * ld[j] + i] = x[r] . row i of w[j]. swiglu == 1: w = {gate, up}
 * of equal rows, out[0][r * ld[0] + i] = silu(g) * u. rows 1..8 FP32 input
 * rows x[r * K + k]. Each call packs the matrices into `workspace`
 * (lfm3_cuda_decode_workspace_bytes, 256-byte aligned) before projecting. */
size_t lfm3_cuda_decode_workspace_bytes(const lfm3_tensor* const* w, int n_w,
                                        int swiglu);
int lfm3_cuda_decode_project(const lfm3_tensor* const* w, int n_w, int swiglu,
                             const float* x, int rows, float* const* out,
                             const size_t* ld, void* workspace, void* stream);
int lfm3_cuda_batched_quant_gemm_fp32(uint32_t type, const void* w,
                                      const float* x, float* y, size_t batch,
                                      size_t m, size_t k, void* stream);
int lfm3_cuda_exact_bf16_gemm_fp32_small_batch(const void* A, const float* X,
                                               float* Y, size_t batch, size_t M,
                                               size_t K, void* stream);

/* LaunchBatchedRMSNorm (hip/ops.hpp:148-150): out = x * rsqrt(mean x^2 +
 * eps) * weight per row (bf16 output not supported: out_bf16 must be NULL). */
int lfm3_cuda_batched_rmsnorm(const float* x, const float* weight, float* out,
                              void* out_bf16, size_t batch, size_t dim,
                              float eps, void* stream);

/* ---- token selection --------------------------------------------------------
 * The reference's runner reads each round's logits to the host and samples
 * them with Gufo core's sampling::SamplerState (runner.cpp:268-296, defaults
 * temperature 0.1, top-k 50, repeat penalty 1.1 at runner.cpp:31-35). That
 * sampler is not in the reference tree; this library's rule, the same on the
 * device and on the host:
 *   1. each distinct token of a row's recent tokens: l = l > 0 ? l / p : l * p
 *   2. the top_k largest logits, ordered by (logit descending, id ascending)
 *   3. w_i = exp((l_i - l_0) / temperature) in double precision, S = w_0 +
 *      w_1 + ... in that order, u = uniform [0, 1) from the row's seed
 *      (SplitMix64), token = first candidate whose running sum exceeds u * S.
 * Temperature 0 selects the largest penalised logit (lowest id on ties).
 * Per-row tables are HOST memory read at call time: recent[r * 64 + j] for
 * j < recent_count[r] (<= 64; the caller's penalty window, e.g. the row's
 * last 64 tokens), seeds[r] (a fresh value per draw, e.g. a hash of the
 * session's seed and position). */
#define LFM3_SAMPLE_MAX_TOP_K 64
#define LFM3_SAMPLE_MAX_RECENT 64
typedef struct lfm3_sampler {
  float temperature;    /* >= 0; 0 selects the largest logit */
  uint32_t top_k;       /* 1..64 (ignored at temperature 0) */
  float repeat_penalty; /* > 0; 1 disables the penalty */
} lfm3_sampler;

/* Device scratch bytes of lfm3_cuda_sample for rows x vocab. */
size_t lfm3_cuda_sample_scratch_bytes(int rows, int vocab, int top_k);
/* Device selection: logits [rows][ld] and tokens[rows] are device memory,
 * the tables host memory; vocab <= 64 x 4096 / top_k. */
int lfm3_cuda_sample(const float* logits, int rows, int vocab, int ld,
                     const lfm3_sampler* sampler, const uint32_t* recent,
                     const uint32_t* recent_count, const uint64_t* seeds,
                     uint32_t* tokens, void* scratch, void* stream);
/* The same selection on the host (host logits and tokens). */
int lfm3_sample_host(const float* logits, int rows, int vocab, int ld,
                     const lfm3_sampler* sampler, const uint32_t* recent,
                     const uint32_t* recent_count, const uint64_t* seeds,
                     uint32_t* tokens);

/* ---- engine (engine.hpp) --------------------------------------------------- */

typedef struct lfm3_model lfm3_model;
typedef struct lfm3_session lfm3_session;

/* Model::Load (engine.hpp:27-30) from host tensors: validates the geometry,
 * copies the packed payloads to the current CUDA device. NULL on failure. */
lfm3_model* lfm3_model_load(const lfm3_weights* host);
void lfm3_model_free(lfm3_model* model);
int lfm3_model_config(const lfm3_model* model, lfm3_config* out);
size_t lfm3_model_weight_bytes(const lfm3_model* model);

/* Model::CreateSession (engine.hpp:31-32). NULL on failure. */
lfm3_session* lfm3_session_create(lfm3_model* model, uint32_t context);
void lfm3_session_free(lfm3_session* session);

/* Session::Forward (engine.hpp:98-101): logits (vocab floats) may be NULL. */
int lfm3_session_forward(lfm3_session* session, const uint32_t* tokens,
                         size_t n, float* logits);
/* Session::ForwardBatch (engine.hpp:103-106): one token per session, up to
 * eight distinct sessions; logits may be NULL or hold NULL entries. */
int lfm3_session_forward_batch(lfm3_session* const* sessions,
                               const uint32_t* tokens, size_t count,
                               float* const* logits);
/* Session::ForwardBatchInputs (engine.hpp:107-114): one row per session;
 * rows (may be NULL) holds per session NULL (tokens[i] is the input) or a
 * device row of hidden input-embedding floats, ready in the calling
 * sessions' stream order (tokens[i] is then ignored). With logits set, each session's logits are computed into its
 * device buffer (lfm3_session_continuation_data tensor 0) without a copy to
 * the host. Returns once the round is queued: work queued on a session's
 * lfm3_session_stream runs after it, the session's reads wait for it, and a
 * device wait that gave up is reported by the next call that waits. */
int lfm3_session_forward_batch_inputs(lfm3_session* const* sessions,
                                      const uint32_t* tokens,
                                      const float* const* rows, size_t count,
                                      int logits);
/* A batched round followed by token selection on the device: the runner's
 * AdvanceBatch + SelectNext (runner.cpp:268-351) without the logits' trip
 * to the host. One token per session in, next[i] (host) the token selected
 * from session i's new logits by `sampler` with row i of the host tables
 * (see lfm3_sampler); the logits also stay readable by
 * lfm3_session_read_logits. Returns after the tokens are on the host. */
int lfm3_session_forward_batch_sample(lfm3_session* const* sessions,
                                      const uint32_t* tokens, size_t count,
                                      const lfm3_sampler* sampler,
                                      const uint32_t* recent,
                                      const uint32_t* recent_count,
                                      const uint64_t* seeds, uint32_t* next);
/* Session::ForwardEmbeddings (engine.hpp:115-120): n rows of hidden
 * input-embedding floats, in host memory, or in device memory read in this
 * session's stream order when on_device is nonzero; logits (host, vocab
 * floats) may be NULL. */
int lfm3_session_forward_embeddings(lfm3_session* session, const float* rows,
                                    size_t n, int on_device, float* logits);
/* Session::Input / ForwardInputs (engine.hpp:121-131): runs of token ids or
 * of host embedding rows (one of the two per run), advanced in order with
 * adjacent runs sharing their 512-row passes. */
typedef struct lfm3_input {
  const uint32_t* tokens;
  size_t n_tokens;
  const float* rows; /* n_rows x hidden floats, host memory */
  size_t n_rows;
} lfm3_input;
int lfm3_session_forward_inputs(lfm3_session* session,
                                const lfm3_input* inputs, size_t count,
                                float* logits);
/* Session::Speculate (engine.hpp:71-73): the reference starts an NPU decode
 * early; the GPU has nothing to start, so this only checks the session. */
int lfm3_session_speculate(lfm3_session* session, uint32_t token);
/* Session::ForwardDecision / ForwardDecisions (engine.hpp:54-70, d1 models
 * with bidirectional attention): not built; returns LFM3_ERR_UNSUPPORTED. */
int lfm3_session_forward_decision(lfm3_session* session,
                                  const uint32_t* tokens, size_t n,
                                  float* logits);
int lfm3_session_read_logits(lfm3_session* session, float* logits);
int lfm3_session_read_hidden(lfm3_session* session, float* hidden);
int lfm3_session_reset(lfm3_session* session);
uint32_t lfm3_session_position(const lfm3_session* session);
int lfm3_session_is_coherent(const lfm3_session* session);
void* lfm3_session_stream(const lfm3_session* session);
/* ContinuationData (engine.hpp:143-144): tensor 0 logits, 1 frontier,
 * 2 convolution, 3 key ring, 4 value ring (device pointers). */
void* lfm3_session_continuation_data(const lfm3_session* session, int tensor,
                                     size_t layer);
uint32_t lfm3_session_ring_capacity(const lfm3_session* session,
                                    size_t layer);
/* ContinuationHooks (continuation_hooks.hpp:5-16) as C callbacks: each
 * runs on the calling thread before the session changes state or submits
 * device work, and refuses it by returning nonzero (the call then fails
 * with LFM3_ERR_INVALID and changes nothing). before_write gets the rows
 * [first, end) about to be written. SetContinuationHooks
 * (engine.hpp:146): hooks is copied; NULL removes them. */
typedef struct lfm3_continuation_hooks {
  void* user;
  int (*before_write)(void* user, uint32_t first, uint32_t end);
  int (*before_reset)(void* user);
  int (*before_restore)(void* user);
} lfm3_continuation_hooks;
int lfm3_session_set_continuation_hooks(lfm3_session* session,
                                        const lfm3_continuation_hooks* hooks);
/* PrepareLogits (engine.hpp:153-154): computes the frontier's logits on the
 * session's stream when the last advance did not. BeginRestore /
 * FinishRestore (engine.hpp:155-156): around direct writes to the
 * continuation buffers; BeginRestore waits for queued work and marks the
 * session incoherent, FinishRestore(position) makes it coherent at
 * `position` with the written frontier and logits. */
int lfm3_session_prepare_logits(lfm3_session* session);
int lfm3_session_begin_restore(lfm3_session* session);
int lfm3_session_finish_restore(lfm3_session* session, uint32_t position);
/* ---- continuous batching ------------------------------------------------
 * The step the reference's host scheduler drives through its text runner
 * (scheduling profile runner.cpp:140-177: prompt passes of at most 512 rows
 * in one layer group between decode rounds of at most 8 sessions; Prefill /
 * AdvanceBatch / SelectNext, runner.cpp:249-351). Each step runs one prompt
 * pass of at most 512 rows for the first admitted request with prompt rows
 * left (first come, first served; after its last pass the request's first
 * token is selected on the device), then one decode round of up to 8
 * decoding requests in admission order with device token selection. Every
 * selection uses the scheduler's sampler over the request's last 64 tokens
 * (prompt tail, then each advanced token) and the draw seed
 * seed ^ (position * 0x9E3779B97F4A7C15), position = tokens advanced.
 * One host thread per scheduler. */
typedef struct lfm3_scheduler lfm3_scheduler;
typedef struct lfm3_step_stats {
  int32_t pass_request; /* request of the step's prompt pass, or -1 */
  uint32_t pass_rows;
  uint32_t round_rows;  /* requests the decode round advanced */
  uint32_t finished;    /* requests completed by the step */
  double pass_ms;       /* host time of the pass (results on the host) */
  double round_ms;      /* host time of the round (tokens on the host) */
} lfm3_step_stats;
lfm3_scheduler* lfm3_scheduler_create(lfm3_model* model,
                                      const lfm3_sampler* sampler);
void lfm3_scheduler_free(lfm3_scheduler* scheduler);
/* Admits a request (the prompt is copied) with its own session of
 * `context` rows (>= n + max_new). Returns the request id (>= 0) or a
 * negative LFM3_ERR_* code. */
int lfm3_scheduler_admit(lfm3_scheduler* scheduler, const uint32_t* prompt,
                         size_t n, uint32_t max_new, uint64_t seed,
                         uint32_t context);
/* One step; stats may be NULL. A failed device call retires the requests
 * of that call (LFM3_ERR_CUDA or LFM3_ERR_DEVICE_WAIT); the others go on. */
int lfm3_scheduler_step(lfm3_scheduler* scheduler, lfm3_step_stats* stats);
/* 1 when no admitted request has work left, else 0. */
int lfm3_scheduler_idle(const lfm3_scheduler* scheduler);
/* The tokens request `id` has selected so far: copies up to cap into out
 * (may be NULL) and returns how many there are. */
size_t lfm3_scheduler_tokens(const lfm3_scheduler* scheduler, int id,
                             uint32_t* out, size_t cap);
/* 1 when request `id` is complete (2 when it was retired by a failure),
 * else 0. */
int lfm3_scheduler_finished(const lfm3_scheduler* scheduler, int id);

/* Snapshot v2 (engine.hpp:127-131). Header word 7 is
 * lfm3_snapshot_signature of the model's configuration. */
size_t lfm3_session_snapshot_bytes(const lfm3_session* session);
/* ConfigSignature (engine.cpp:1403-1419): FNV-1a over hidden, intermediate,
 * vocab, heads, head_dim, window, conv_width, the bit patterns of eps, theta
 * and theta_swa, then each layer's type and KV head count. Host only. */
uint32_t lfm3_snapshot_signature(const lfm3_config* config);
int lfm3_session_save_snapshot(lfm3_session* session, uint8_t* out,
                               size_t bytes);
int lfm3_session_restore_snapshot(lfm3_session* session, const uint8_t* data,
                                  size_t bytes);
/* Test hook (no reference counterpart): the k-th CUDA call of this
 * session's next passes reports a failure, to exercise poisoning. */
int lfm3_session_inject_failure(lfm3_session* session, int after_calls);

/* Measurement hooks (no reference counterpart). With profiling on, CUDA
 * events bracket every kernel of this session's passes (and of rounds it
 * leads), which serialises them: use a separate profiled pass. take_profile
 * adds the milliseconds and launch counts of the 6 kernel classes (decode
 * projection, decode attention, row kernels, prompt projection, prompt
 * attention, other prompt kernels) to ms[6] / launches[6] and clears them. */
int lfm3_session_set_profiling(lfm3_session* session, int on);
int lfm3_session_take_profile(lfm3_session* session, double* ms,
                              long long* launches);
/* Kernels launched by this library in this process so far. */
unsigned long long lfm3_cuda_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif
