// extern "C" entry points of include/lfm3_cuda.h: the operator surface of
// hip/ops.hpp and the engine of engine.hpp over this library's kernels.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "../../include/lfm3_cuda.h"
#include "common.cuh"
#include "engine.hpp"
#include "kernels.cuh"
#include "scheduler.hpp"

namespace {

thread_local std::string g_last_error;

int Fail(int code, const std::string& message) {
  g_last_error = message;
  return code;
}
int Cuda(cudaError_t e) {
  if (e == cudaSuccess)
    return LFM3_OK;
  return Fail(e == cudaErrorInvalidValue ? LFM3_ERR_UNSUPPORTED : LFM3_ERR_CUDA,
              cudaGetErrorString(e));
}
cudaStream_t Stream(void* s) { return static_cast<cudaStream_t>(s); }

int Sms() {
  static thread_local int device = -1, count = 148;
  int current = 0;
  if (cudaGetDevice(&current) == cudaSuccess && current != device) {
    device = current;
    cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, current);
  }
  return count;
}

constexpr int kPromptRows = 16;  // hip/ops.hpp:33
constexpr size_t kTicketWords = 8192;

bool Q8Matrix(const lfm3_tensor* t) {
  return t && t->data && t->type == LFM3_Q8_0 && t->cols % 512 == 0;
}
bool Bf16Matrix(const lfm3_tensor* t) {
  return t && t->data && t->type == LFM3_BF16 && t->cols % 256 == 0;
}

// BF16 projections of any number of FP32 rows (exact BF16 x FP32 on the
// CUDA cores; hip/ops.hip:1917-2005).
int Bf16Rows(lfm3::GemvParams p, const float* x, int n, int K,
             cudaStream_t s) {
  p.K = K;
  if (!lfm3::bf16_plan(p))
    return Fail(LFM3_ERR_UNSUPPORTED, "BF16 projection width not tiled");
  return Cuda(lfm3::launch_bf16_gemv(p, x, K, n, s));
}

// Decode projections of n < 16 FP32 rows: split once, then <= 8 rows per
// launch.
int GemvRows(lfm3::GemvParams p, const float* x, int n, int K,
             const lfm3_dense_workspace& ws, cudaStream_t s,
             std::vector<size_t> out_row_stride) {
  if (!ws.quantized)
    return Fail(LFM3_ERR_INVALID, "workspace needs quantized");
  p.K = K;
  if (!lfm3::gemv_plan(p, Sms()))
    return Fail(LFM3_ERR_UNSUPPORTED, "projection width not tiled");
  if (int e = Cuda(lfm3::launch_split_rows(x, ws.quantized, n, K, s)))
    return e;
  if (int e = Cuda(lfm3::fill_gemv_maps(p)))
    return e;
  const int grid = lfm3::gemv_grid(p.tiles, Sms());
  for (int r0 = 0; r0 < n; r0 += lfm3::kMaxBatch) {
    lfm3::GemvParams q = p;
    q.tokens = std::min(lfm3::kMaxBatch, n - r0);
    q.x = static_cast<const char*>(ws.quantized) + size_t(r0) * K * 4;
    for (int j = 0; j < p.n_out; ++j)
      if (q.o[j].out)
        q.o[j].out += size_t(r0) * out_row_stride[j];
    if (int e = Cuda(lfm3::launch_q8_gemv(q, grid, s, false)))
      return e;
  }
  return LFM3_OK;
}

// Prompt projections of n >= 16 rows: FP16 row-scaled input.
int PrefillRows(lfm3::PrefillParams p, const float* x, int n, int K,
                const lfm3_dense_workspace& ws, cudaStream_t s,
                bool split_ready) {
  if (!ws.quantized)
    return Fail(LFM3_ERR_INVALID, "workspace needs quantized");
  auto* values = static_cast<__half*>(ws.quantized);
  auto* scale = reinterpret_cast<float*>(values + size_t(n) * K);
  if (!split_ready)
    if (int e = Cuda(lfm3::launch_half_rows(x, nullptr, values, scale, n, K, s)))
      return e;
  p.K = K;
  p.tokens = n;
  p.x_row0 = 0;
  p.scale = scale;
  // split-K partial sums when the caller passed the split workspace
  p.partial = ws.partial;
  return Cuda(lfm3::launch_q8_prefill(p, values, n, s));
}

int ProjectImpl(const lfm3_output* outputs, int count, const float* x, int n,
                cudaStream_t s, const lfm3_dense_workspace* ws,
                bool split_ready) {
  if (!outputs || count < 1 || count > 4 || n < 0 || !ws)
    return Fail(LFM3_ERR_INVALID, "invalid projection arguments");
  if (n == 0)
    return LFM3_OK;
  const uint32_t K = outputs[0].weight ? outputs[0].weight->cols : 0;
  const bool bf16 = Bf16Matrix(outputs[0].weight);
  for (int j = 0; j < count; ++j)
    if (!(bf16 ? Bf16Matrix(outputs[j].weight) : Q8Matrix(outputs[j].weight)) ||
        outputs[j].weight->cols != K || !outputs[j].out)
      return Fail(LFM3_ERR_UNSUPPORTED,
                  "projections need Q8_0 (widths multiples of 512) or BF16 "
                  "(multiples of 256) weights of one type and width");
  if (bf16) {
    lfm3::GemvParams p{};
    p.kind = lfm3::kGemvPlain;
    p.n_out = count;
    for (int j = 0; j < count; ++j) {
      const auto* w = outputs[j].weight;
      p.o[j] = {static_cast<const uint8_t*>(w->data), outputs[j].out,
                int(w->rows), int(w->rows)};
    }
    return Bf16Rows(p, x, n, int(K), s);
  }
  if (n < kPromptRows) {
    lfm3::GemvParams p{};
    p.kind = lfm3::kGemvPlain;
    p.n_out = count;
    std::vector<size_t> strides;
    for (int j = 0; j < count; ++j) {
      const auto* w = outputs[j].weight;
      p.o[j] = {static_cast<const uint8_t*>(w->data), outputs[j].out,
                int(w->rows), int(w->rows)};
      strides.push_back(w->rows);
    }
    return GemvRows(p, x, n, int(K), *ws, s, strides);
  }
  lfm3::PrefillParams p{};
  p.kind = lfm3::kPrefillPlain;
  p.n_out = count;
  for (int j = 0; j < count; ++j) {
    const auto* w = outputs[j].weight;
    p.o[j] = {static_cast<const uint8_t*>(w->data), outputs[j].out,
              int(w->rows), int(w->rows)};
  }
  return PrefillRows(p, x, n, int(K), *ws, s, split_ready);
}

// ---- small utility kernels -----------------------------------------------------
__global__ void rope_kernel(float* x, const float* frequencies,
                            const float* factors, int n, int heads, int dim,
                            int position) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int pairs = dim / 2;
  if (i >= n * heads * pairs)
    return;
  const int pair = i % pairs, head = i / pairs, row = head / heads;
  float angle = float(position + row) * frequencies[pair];
  if (factors)
    angle /= factors[pair];
  float sn, cs;
  sincosf(angle, &sn, &cs);
  float* h = x + size_t(head) * dim;
  const float a = h[pair], b = h[pair + pairs];
  h[pair] = a * cs - b * sn;
  h[pair + pairs] = b * cs + a * sn;
}

__global__ void pack_kernel(const float* k, const float* v, __half* k16,
                            __half* v16, size_t count) {
  const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= count)
    return;
  k16[i] = __float2half_rn(k[i]);
  v16[i] = __float2half_rn(v[i]);
}

__global__ void copy_rows_kernel(const unsigned char* source,
                                 const uint32_t* rows, unsigned char* out,
                                 size_t bytes) {
  const size_t row = blockIdx.x;
  for (size_t i = threadIdx.x; i < bytes; i += blockDim.x)
    out[row * bytes + i] = source[size_t(rows[row]) * bytes + i];
}

// One matrix times rows of FP32 x through the Dense path, with the Q8_0
// input workspace in stream-ordered memory.
int MatrixRows(const void* w, uint32_t type, const float* x, float* y,
               size_t rows, size_t M, size_t K, cudaStream_t s) {
  if (!w || !x || !y || !rows || !M || !K || rows > size_t(1) << 24 ||
      M > UINT32_MAX || K > UINT32_MAX)
    return Fail(LFM3_ERR_INVALID, "invalid matrix arguments");
  const size_t row_bytes =
      type == LFM3_Q8_0 ? K / 32 * 34 : type == LFM3_BF16 ? K * 2 : 0;
  if (!row_bytes)
    return Fail(LFM3_ERR_UNSUPPORTED, "matrices must be Q8_0 or BF16");
  const lfm3_tensor t{w, type, uint32_t(K), uint32_t(M), M * row_bytes};
  const lfm3_output o{&t, y};
  lfm3_dense_workspace ws{};
  if (type == LFM3_BF16 && !Bf16Matrix(&t))
    return Fail(LFM3_ERR_UNSUPPORTED, "BF16 width must be a multiple of 256");
  if (type == LFM3_Q8_0) {
    if (!Q8Matrix(&t))
      return Fail(LFM3_ERR_UNSUPPORTED, "Q8_0 width must be a multiple of 512");
    if (const int e = Cuda(cudaMallocAsync(
            &ws.quantized, lfm3_cuda_dense_workspace_bytes(rows, K), s)))
      return e;
  }
  int rc = ProjectImpl(&o, 1, x, int(rows), s, &ws, false);
  if (ws.quantized) {
    const int e = Cuda(cudaFreeAsync(ws.quantized, s));
    if (rc == LFM3_OK)
      rc = e;
  }
  return rc;
}

// Controls and per-row tables checked for `rows` rows of `vocab` logits.
int SampleArgs(const lfm3_sampler* sampler, int rows, int vocab,
               const uint32_t* recent, const uint32_t* recent_count,
               const uint64_t* seeds, lfm3::SampleControls* c) {
  if (!sampler || rows < 1 || !recent_count || !seeds || !recent)
    return Fail(LFM3_ERR_INVALID, "sampler, rows and row tables required");
  if (const char* why = lfm3::sample_controls(
          sampler->temperature, sampler->top_k, sampler->repeat_penalty,
          vocab, c))
    return Fail(LFM3_ERR_INVALID, why);
  for (int r = 0; r < rows; ++r) {
    if (recent_count[r] > uint32_t(lfm3::kSampleMaxRecent))
      return Fail(LFM3_ERR_INVALID, "more than 64 recent tokens in a row");
    for (uint32_t j = 0; j < recent_count[r]; ++j)
      if (recent[size_t(r) * lfm3::kSampleMaxRecent + j] >= uint32_t(vocab))
        return Fail(LFM3_ERR_INVALID, "recent token outside the vocabulary");
  }
  return LFM3_OK;
}

}  // namespace

int lfm3::set_last_error(int code, const char* message) {
  return Fail(code, message);
}

extern "C" {

const char* lfm3_last_error(void) { return g_last_error.c_str(); }

unsigned lfm3_cuda_take_device_error(void) { return lfm3::take_device_error(); }

int lfm3_cuda_wait_probe(unsigned limit_us, void* stream) {
  if (limit_us == 0 || limit_us > 1000000)
    return lfm3::set_last_error(LFM3_ERR_INVALID,
                                "wait probe limit must be 1..1000000 us");
  return Cuda(lfm3::launch_wait_probe(uint64_t(limit_us) * 1000,
                                      Stream(stream)));
}

size_t lfm3_cuda_dense_workspace_bytes(size_t rows, size_t K) {
  // FP16 prompt rows + scales, or split decode rows (4 bytes per element)
  return std::max(rows * K * 2 + rows * 4, rows * K * 4);
}
size_t lfm3_cuda_split_partial_bytes(void) {
  // prompt projections with few tiles split K (decode projections never do)
  return lfm3::kPrefillPartialFloats * sizeof(float);
}
size_t lfm3_cuda_split_ticket_words(void) { return kTicketWords; }
int lfm3_cuda_prompt_rows(void) { return kPromptRows; }

int lfm3_cuda_embed(const lfm3_tensor* weight, const uint32_t* tokens,
                    float* out, int n, void* stream) {
  if (!weight || !weight->data || !tokens || !out || n < 0)
    return Fail(LFM3_ERR_INVALID, "invalid embed arguments");
  return Cuda(lfm3::launch_embed_norm(weight->data, weight->type, tokens,
                                      nullptr, out, nullptr, lfm3::NormOut{}, n,
                                      int(weight->cols), 0, Stream(stream),
                                      false));
}

int lfm3_cuda_dense(const lfm3_tensor* weight, const float* x, float* out,
                    int n, void* stream, const lfm3_dense_workspace* workspace) {
  const lfm3_output o{weight, out};
  return ProjectImpl(&o, 1, x, n, Stream(stream), workspace, false);
}

int lfm3_cuda_project(const lfm3_output* outputs, int count, const float* x,
                      int n, void* stream,
                      const lfm3_dense_workspace* workspace, int split_ready) {
  return ProjectImpl(outputs, count, x, n, Stream(stream), workspace,
                     split_ready != 0);
}

int lfm3_cuda_project_swiglu(const lfm3_tensor* gate, const lfm3_tensor* up,
                             const float* x, float* out, float* up_scratch,
                             int n, void* stream,
                             const lfm3_dense_workspace* ws, int split_ready) {
  (void)up_scratch;  // the fused kernels keep up x in registers
  const bool bf16 = Bf16Matrix(gate) && Bf16Matrix(up);
  if (!(bf16 || (Q8Matrix(gate) && Q8Matrix(up))) || gate->rows != up->rows ||
      gate->cols != up->cols || !out || !ws || n < 0)
    return Fail(LFM3_ERR_UNSUPPORTED, "invalid SwiGLU projection");
  if (n == 0)
    return LFM3_OK;
  const cudaStream_t s = Stream(stream);
  const int K = int(gate->cols);
  if (bf16) {
    lfm3::GemvParams p{};
    p.kind = lfm3::kGemvSwiGLU;
    p.n_out = 2;
    p.o[0] = {static_cast<const uint8_t*>(gate->data), out, int(gate->rows),
              int(gate->rows)};
    p.o[1] = {static_cast<const uint8_t*>(up->data), nullptr, int(up->rows),
              0};
    return Bf16Rows(p, x, n, K, s);
  }
  if (n < kPromptRows) {
    lfm3::GemvParams p{};
    p.kind = lfm3::kGemvSwiGLU;
    p.n_out = 2;
    p.o[0] = {static_cast<const uint8_t*>(gate->data), out, int(gate->rows),
              int(gate->rows)};
    p.o[1] = {static_cast<const uint8_t*>(up->data), nullptr, int(up->rows),
              0};
    return GemvRows(p, x, n, K, *ws, s, {gate->rows, 0});
  }
  if (ws->row_max)
    if (int e = Cuda(cudaMemsetAsync(ws->row_max, 0, size_t(n) * 4, s)))
      return e;
  lfm3::PrefillParams p{};
  p.kind = lfm3::kPrefillSwiGLU;
  p.n_out = 2;
  p.o[0] = {static_cast<const uint8_t*>(gate->data), out, int(gate->rows),
            int(gate->rows)};
  p.o[1] = {static_cast<const uint8_t*>(up->data), nullptr, int(up->rows), 0};
  p.row_max = ws->row_max;
  return PrefillRows(p, x, n, K, *ws, s, split_ready != 0);
}

int lfm3_cuda_project_ffn(const lfm3_tensor* gate, const lfm3_tensor* up,
                          const lfm3_tensor* down, const float* x,
                          float* hidden, float* up_scratch, float* out, int n,
                          void* stream, const lfm3_dense_workspace* ws,
                          int split_ready) {
  if (!(Q8Matrix(down) || Bf16Matrix(down)) || !gate ||
      down->cols != gate->rows || down->type != gate->type)
    return Fail(LFM3_ERR_UNSUPPORTED, "invalid FFN down projection");
  if (int e = lfm3_cuda_project_swiglu(gate, up, x, hidden, up_scratch, n,
                                       stream, ws, split_ready))
    return e;
  if (n >= kPromptRows && ws->row_max && down->type == LFM3_Q8_0) {
    // down input from the SwiGLU row maxima (HalfRowsFromMax)
    auto* values = static_cast<__half*>(ws->quantized);
    auto* scale = reinterpret_cast<float*>(values + size_t(n) * down->cols);
    if (int e = Cuda(lfm3::launch_half_rows(hidden, ws->row_max, values, scale,
                                            n, int(down->cols),
                                            Stream(stream))))
      return e;
    const lfm3_output o{down, out};
    return ProjectImpl(&o, 1, hidden, n, Stream(stream), ws, true);
  }
  return lfm3_cuda_dense(down, hidden, out, n, stream, ws);
}

int lfm3_cuda_residual_norm(const float* branch, const lfm3_tensor* post_norm,
                            float* x, const lfm3_tensor* norm, float* z, int n,
                            int hidden, float eps, int split, void* stream,
                            const lfm3_dense_workspace* ws) {
  if (hidden % 256 || hidden > 8192)
    return Fail(LFM3_ERR_UNSUPPORTED, "unsupported residual-norm width");
  if (!x || n < 0 || (split && (!ws || !ws->quantized)))
    return Fail(LFM3_ERR_INVALID, "invalid residual-norm arguments");
  lfm3::NormOut out{};
  if (split) {
    out.half = static_cast<__half*>(ws->quantized);
    out.scale = reinterpret_cast<float*>(out.half + size_t(n) * hidden);
  } else {
    out.f32 = z;
  }
  return Cuda(lfm3::launch_residual_norm(
      branch,
      post_norm && post_norm->data ? static_cast<const float*>(post_norm->data)
                                   : nullptr,
      x, norm ? static_cast<const float*>(norm->data) : nullptr, out, n, hidden,
      eps, Stream(stream), false));
}

int lfm3_cuda_short_conv(const float* projection, const float* weight,
                         float* history, float* out, int n, int hidden,
                         int width, void* stream, int update) {
  if (!projection || !weight || !history || !out)
    return Fail(LFM3_ERR_INVALID, "invalid convolution arguments");
  return Cuda(lfm3::launch_short_conv(projection, weight, history, out, n,
                                      hidden, width, update != 0,
                                      Stream(stream)));
}

int lfm3_cuda_rope_frequencies(float* out, int dim, float theta, void* stream) {
  if (!out || dim <= 0 || dim % 2 || dim > 1024)
    return Fail(LFM3_ERR_INVALID, "invalid RoPE dimension");
  float host[512];
  for (int i = 0; i < dim / 2; ++i)
    host[i] = float(std::pow(double(theta), double(-2.0F * i / dim)));
  return Cuda(cudaMemcpyAsync(out, host, size_t(dim / 2) * 4,
                              cudaMemcpyHostToDevice, Stream(stream)));
}

int lfm3_cuda_rope(float* x, const float* frequencies, const float* factors,
                   int n, int heads, int dim, int position, void* stream) {
  if (!x || !frequencies || dim % 2 || n < 0 || heads <= 0)
    return Fail(LFM3_ERR_INVALID, "invalid RoPE arguments");
  const int total = n * heads * (dim / 2);
  if (!total)
    return LFM3_OK;
  rope_kernel<<<(total + 255) / 256, 256, 0, Stream(stream)>>>(
      x, frequencies, factors, n, heads, dim, position);
  return Cuda(cudaGetLastError());
}

size_t lfm3_cuda_attention_scratch_bytes(int heads, int dim, int context,
                                         int rows) {
  (void)dim;
  const size_t decode = lfm3::decode_attention_partial_floats(heads) * 4 +
                        lfm3::kMaxBatch * 64 * 4;  // partials + tickets
  const size_t prompt =
      lfm3::prompt_attention_scratch_floats(heads, rows, context) * 4;
  return std::max(decode, prompt);
}

int lfm3_cuda_attention(const float* q, const uint16_t* k, const uint16_t* v,
                        const float* gate, const uint16_t* cache_k,
                        const uint16_t* cache_v, float* out, int n, int heads,
                        int kv_heads, int dim, int position, int capacity,
                        int window, void* stream, float* scratch) {
  if (dim != 128 || kv_heads <= 0 || heads % kv_heads ||
      (heads / kv_heads != 2 && heads / kv_heads != 4 && heads / kv_heads != 8))
    return Fail(LFM3_ERR_UNSUPPORTED, "unsupported LFM3 attention shape");
  if (!q || !k || !v || !gate || !out || !scratch || n < 0 || capacity <= 0)
    return Fail(LFM3_ERR_INVALID, "invalid attention arguments");
  const cudaStream_t s = Stream(stream);
  const auto* hk = reinterpret_cast<const __half*>(k);
  const auto* hv = reinterpret_cast<const __half*>(v);
  const auto* ck = reinterpret_cast<const __half*>(cache_k);
  const auto* cv = reinterpret_cast<const __half*>(cache_v);
  if (n == 1) {
    lfm3::DecodeAttentionParams p{};
    p.q = q;
    p.gate = gate;
    p.ldq = heads * 128;
    p.ldg = heads;
    p.heads = heads;
    p.kv_heads = kv_heads;
    p.window = window;
    p.max_splits = lfm3::kMaxDecodeSplits;
    p.out_f32 = out;
    p.partials = scratch;
    // tickets live after the partials, zeroed here (they return to zero)
    auto* tickets = reinterpret_cast<unsigned*>(
        scratch + lfm3::decode_attention_partial_floats(heads));
    if (int e = Cuda(cudaMemsetAsync(tickets, 0, lfm3::kMaxBatch * 64 * 4, s)))
      return e;
    p.tickets = tickets;
    p.position = position;
    p.ring_k = ck;
    p.ring_v = cv;
    p.chunk_k = hk;
    p.chunk_v = hv;
    p.capacity = capacity;
    return Cuda(lfm3::launch_decode_attention(p, 1, s, false));
  }
  return Cuda(lfm3::launch_prompt_attention(
      q, heads * 128, hk, hv, ck, cv, gate, heads, out, n, heads, kv_heads,
      position, capacity, window, scratch, s));
}

int lfm3_cuda_attention_stored(const float* q, const float* gate,
                               const uint16_t* cache_k,
                               const uint16_t* cache_v, float* out, int n,
                               int heads, int kv_heads, int dim, int position,
                               int capacity, void* stream, float* scratch) {
  if (dim != 128 || kv_heads <= 0 || heads % kv_heads ||
      (heads / kv_heads != 2 && heads / kv_heads != 4 && heads / kv_heads != 8))
    return Fail(LFM3_ERR_UNSUPPORTED, "unsupported LFM3 attention shape");
  if (!q || !gate || !cache_k || !cache_v || !out || !scratch || n <= 0 ||
      position < 0 || position + n > capacity)
    return Fail(LFM3_ERR_INVALID, "invalid stored-key attention arguments");
  return Cuda(lfm3::launch_prompt_attention_tc(
      q, heads * 128, reinterpret_cast<const __half*>(cache_k),
      reinterpret_cast<const __half*>(cache_v), gate, heads, out, n, heads,
      kv_heads, position, capacity, scratch, Stream(stream)));
}

int lfm3_cuda_prompt_heads(float* q, float* k, const float* v,
                           const float* q_norm, const float* k_norm,
                           const float* frequencies, const float* factors,
                           uint16_t* k16, uint16_t* v16, int n, int heads,
                           int kv_heads, int dim, int position, float eps,
                           void* stream) {
  if (dim != 128)
    return Fail(LFM3_ERR_UNSUPPORTED, "LFM3 prompt heads need dimension 128");
  return Cuda(lfm3::launch_prompt_heads(
      q, k, v, heads * 128, kv_heads * 128, q_norm, k_norm, frequencies,
      factors, reinterpret_cast<__half*>(k16), reinterpret_cast<__half*>(v16),
      n, heads, kv_heads, position, eps, Stream(stream)));
}

int lfm3_cuda_decode_heads(float* q, float* k, const float* v,
                           const float* q_norm, const float* k_norm,
                           const float* frequencies, const float* factors,
                           uint16_t* cache_k, uint16_t* cache_v, int heads,
                           int kv_heads, int dim, int position, int capacity,
                           float eps, void* stream) {
  if (dim != 128)
    return Fail(LFM3_ERR_UNSUPPORTED, "LFM3 decode heads need dimension 128");
  if (capacity <= 0)
    return Fail(LFM3_ERR_INVALID, "invalid ring capacity");
  const size_t slot = size_t(position % capacity) * kv_heads * 128;
  return Cuda(lfm3::launch_prompt_heads(
      q, k, v, heads * 128, kv_heads * 128, q_norm, k_norm, frequencies,
      factors, reinterpret_cast<__half*>(cache_k) + slot,
      reinterpret_cast<__half*>(cache_v) + slot, 1, heads, kv_heads, position,
      eps, Stream(stream)));
}

int lfm3_cuda_store_kv(const uint16_t* k, const uint16_t* v, uint16_t* cache_k,
                       uint16_t* cache_v, int n, int stride, int position,
                       int capacity, void* stream) {
  if (capacity <= 0 || stride <= 0)
    return Fail(LFM3_ERR_INVALID, "invalid ring");
  return Cuda(lfm3::launch_store_kv(
      reinterpret_cast<const __half*>(k), reinterpret_cast<const __half*>(v),
      reinterpret_cast<__half*>(cache_k), reinterpret_cast<__half*>(cache_v), n,
      stride, position, capacity, Stream(stream)));
}

int lfm3_cuda_pack_kv(const float* k, const float* v, uint16_t* k16,
                      uint16_t* v16, size_t count, void* stream) {
  if (!count)
    return LFM3_OK;
  pack_kernel<<<(count + 255) / 256, 256, 0, Stream(stream)>>>(
      k, v, reinterpret_cast<__half*>(k16), reinterpret_cast<__half*>(v16),
      count);
  return Cuda(cudaGetLastError());
}

int lfm3_cuda_select_rows(const lfm3_tensor* source, const uint32_t* rows,
                          void* out, int count, void* stream) {
  if (!source || !source->data || !source->rows || !rows || !out || count < 0)
    return Fail(LFM3_ERR_INVALID, "invalid row selection");
  if (!count)
    return LFM3_OK;
  copy_rows_kernel<<<count, 256, 0, Stream(stream)>>>(
      static_cast<const unsigned char*>(source->data), rows,
      static_cast<unsigned char*>(out), source->bytes / source->rows);
  return Cuda(cudaGetLastError());
}

int lfm3_cuda_batched_rmsnorm(const float* x, const float* weight, float* out,
                              void* out_bf16, size_t batch, size_t dim,
                              float eps, void* stream) {
  if (out_bf16)
    return Fail(LFM3_ERR_UNSUPPORTED, "bf16 norm output is not built");
  if (dim % 256 || dim > 8192 || !x || !weight || !out)
    return Fail(LFM3_ERR_UNSUPPORTED, "unsupported RMSNorm width");
  // residual_norm normalises x in place only when a branch is added; with no
  // branch it reads x and writes out
  return Cuda(lfm3::launch_residual_norm(
      nullptr, nullptr, const_cast<float*>(x), weight,
      lfm3::NormOut{out, nullptr, nullptr, nullptr}, int(batch), int(dim), eps,
      Stream(stream), false));
}

// ---- launch-level operators ---------------------------------------------------------
int lfm3_cuda_shares_split(const lfm3_output* outputs, int count, int n,
                           const lfm3_dense_workspace* workspace) {
  if (!outputs || count < 1 || count > 4 || n < kPromptRows || !workspace ||
      !workspace->quantized)
    return 0;
  for (int j = 0; j < count; ++j)
    if (!Q8Matrix(outputs[j].weight) ||
        outputs[j].weight->cols != outputs[0].weight->cols)
      return 0;
  return 1;
}

int lfm3_cuda_batched_residual_add(const float* a, const float* b, float* out,
                                   size_t batch, size_t dim, void* stream) {
  if (!a || !b || !out)
    return Fail(LFM3_ERR_INVALID, "null argument");
  if (dim % 8 || dim > 8192 || batch > size_t(INT32_MAX))
    return Fail(LFM3_ERR_UNSUPPORTED, "residual add width must be a multiple of 8, <= 8192");
  if (!batch || !dim)
    return LFM3_OK;
  if (out != a)
    if (const int e = Cuda(cudaMemcpyAsync(out, a, batch * dim * 4,
                                           cudaMemcpyDeviceToDevice,
                                           Stream(stream))))
      return e;
  // the residual-norm kernel's plain add (no branch norm, no output norm)
  return Cuda(lfm3::launch_residual_norm(b, nullptr, out, nullptr,
                                         lfm3::NormOut{}, int(batch), int(dim),
                                         0.0F, Stream(stream), false));
}

namespace {
// The decode layout of caller matrices for lfm3_cuda_decode_project, and the
// workspace pieces: packed copy, split input.
struct DecodeWorkspace {
  lfm3::DecodeLayout layout{};
  size_t packed = 0, split = 0, total = 0;
};
bool DecodePlan(const lfm3_tensor* const* w, int n_w, int swiglu,
                DecodeWorkspace& ws) {
  if (!w || n_w < 1 || n_w > 4 || (swiglu && n_w != 2))
    return false;
  auto& l = ws.layout;
  l.kind = swiglu ? lfm3::kDecSwiGLU : lfm3::kDecPlain;
  l.n_src = n_w;
  for (int j = 0; j < n_w; ++j) {
    if (!w[j] || !w[j]->data ||
        (w[j]->type != LFM3_Q8_0 && w[j]->type != LFM3_BF16) ||
        (j && (w[j]->cols != w[0]->cols || w[j]->type != w[0]->type)))
      return false;
    l.rows[j] = int(w[j]->rows);
  }
  l.K = int(w[0]->cols);
  l.bf16 = w[0]->type == LFM3_BF16 ? 1 : 0;
  if (!lfm3::decode_layout(l, Sms()))
    return false;
  const auto up = [](size_t b) { return (b + 255) / 256 * 256; };
  ws.packed = up(lfm3::decode_packed_bytes(l));
  ws.split = up(size_t(lfm3::kMaxBatch) * l.K * 4);
  ws.total = ws.packed + ws.split;
  return true;
}
}  // namespace

size_t lfm3_cuda_decode_workspace_bytes(const lfm3_tensor* const* w, int n_w,
                                        int swiglu) {
  DecodeWorkspace ws;
  return DecodePlan(w, n_w, swiglu, ws) ? ws.total : 0;
}

int lfm3_cuda_decode_project(const lfm3_tensor* const* w, int n_w, int swiglu,
                             const float* x, int rows, float* const* out,
                             const size_t* ld, void* workspace, void* stream) {
  DecodeWorkspace ws;
  if (!DecodePlan(w, n_w, swiglu, ws))
    return Fail(LFM3_ERR_UNSUPPORTED, "decode projection shape not supported");
  if (!x || !out || !ld || !workspace || rows < 1 || rows > lfm3::kMaxBatch ||
      reinterpret_cast<uintptr_t>(workspace) % 256)
    return Fail(LFM3_ERR_INVALID, "invalid decode projection arguments");
  for (int j = 0; j < (swiglu ? 1 : n_w); ++j)
    if (!out[j])
      return Fail(LFM3_ERR_INVALID, "null output");
  cudaStream_t s = Stream(stream);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  uint8_t* packed = base;
  void* split = base + ws.packed;
  const uint8_t* src[4] = {};
  for (int j = 0; j < n_w; ++j)
    src[j] = static_cast<const uint8_t*>(w[j]->data);
  if (int e = Cuda(lfm3::launch_decode_pack(ws.layout, src, packed, s)))
    return e;
  if (int e = Cuda(lfm3::launch_split_rows(x, split, rows, ws.layout.K, s)))
    return e;
  lfm3::DecodeParams p{};
  p.layout = ws.layout;
  p.w = packed;
  p.tokens = rows;
  p.x = split;
  for (int j = 0; j < (swiglu ? 0 : n_w); ++j)
    p.o[j] = lfm3::DecodeOut{out[j], int(ld[j])};
  if (swiglu) {
    p.f32_out = out[0];
    p.f32_ld = int(ld[0]);
  }
  return Cuda(lfm3::launch_decode_gemv(
      p, lfm3::decode_grid(ws.layout, Sms()), s, false));
}

int lfm3_cuda_gemv(const void* A, uint32_t a_type, const float* x, float* y,
                   size_t M, size_t K, void* stream) {
  return MatrixRows(A, a_type, x, y, 1, M, K, Stream(stream));
}

int lfm3_cuda_batched_quant_gemm_fp32(uint32_t type, const void* w,
                                      const float* x, float* y, size_t batch,
                                      size_t m, size_t k, void* stream) {
  if (type != LFM3_Q8_0)
    return Fail(LFM3_ERR_UNSUPPORTED, "quantized matrices must be Q8_0");
  return MatrixRows(w, type, x, y, batch, m, k, Stream(stream));
}

int lfm3_cuda_exact_bf16_gemm_fp32_small_batch(const void* A, const float* X,
                                               float* Y, size_t batch, size_t M,
                                               size_t K, void* stream) {
  return MatrixRows(A, LFM3_BF16, X, Y, batch, M, K, Stream(stream));
}

// ---- token selection ------------------------------------------------------------
size_t lfm3_cuda_sample_scratch_bytes(int rows, int vocab, int top_k) {
  if (rows < 1 || vocab < 1 || top_k < 1)
    return 0;
  return lfm3::sample_scratch_bytes(std::min(rows, 8), vocab,
                                    std::min(top_k, lfm3::kSampleMaxTopK));
}

int lfm3_cuda_sample(const float* logits, int rows, int vocab, int ld,
                     const lfm3_sampler* sampler, const uint32_t* recent,
                     const uint32_t* recent_count, const uint64_t* seeds,
                     uint32_t* tokens, void* scratch, void* stream) {
  lfm3::SampleControls c{};
  if (const int e =
          SampleArgs(sampler, rows, vocab, recent, recent_count, seeds, &c))
    return e;
  if (!logits || !tokens || !scratch || ld < vocab)
    return Fail(LFM3_ERR_INVALID, "logits, tokens and scratch required");
  // eight rows per launch pair, reusing the scratch in stream order
  for (int r0 = 0; r0 < rows; r0 += 8) {
    lfm3::SampleParams p{};
    p.rows = std::min(8, rows - r0);
    p.logits = logits + size_t(r0) * ld;
    p.vocab = vocab;
    p.ld = ld;
    p.segments = (vocab + lfm3::kSampleSegment - 1) / lfm3::kSampleSegment;
    p.c = c;
    for (int r = 0; r < p.rows; ++r) {
      p.recent_count[r] = recent_count[r0 + r];
      p.seed[r] = seeds[r0 + r];
      std::memcpy(p.recent[r], recent + size_t(r0 + r) * lfm3::kSampleMaxRecent,
                  p.recent_count[r] * sizeof(uint32_t));
    }
    p.cand_key = static_cast<uint32_t*>(scratch);
    p.cand_id = p.cand_key + size_t(p.rows) * p.segments * c.top_k;
    p.out = tokens + r0;
    if (const int e = Cuda(lfm3::launch_sample(p, Stream(stream))))
      return e;
  }
  return LFM3_OK;
}

int lfm3_sample_host(const float* logits, int rows, int vocab, int ld,
                     const lfm3_sampler* sampler, const uint32_t* recent,
                     const uint32_t* recent_count, const uint64_t* seeds,
                     uint32_t* tokens) {
  lfm3::SampleControls c{};
  if (const int e =
          SampleArgs(sampler, rows, vocab, recent, recent_count, seeds, &c))
    return e;
  if (!logits || !tokens || ld < vocab)
    return Fail(LFM3_ERR_INVALID, "logits and tokens required");
  lfm3::sample_host(logits, rows, vocab, size_t(ld), c, recent, recent_count,
                    seeds, tokens);
  return LFM3_OK;
}

// ---- engine ---------------------------------------------------------------------
struct lfm3_model {
  std::shared_ptr<lfm3::Model> model;
};
// C callbacks behind the engine's ContinuationHooks: a nonzero return
// refuses the change (the engine call fails before touching the session).
class CHooks final : public lfm3::ContinuationHooks {
public:
  explicit CHooks(const lfm3_continuation_hooks& c) : c_(c) {}
  void BeforeWrite(uint32_t first, uint32_t end) override {
    if (c_.before_write && c_.before_write(c_.user, first, end))
      throw std::runtime_error("continuation hook refused the write");
  }
  void BeforeReset() override {
    if (c_.before_reset && c_.before_reset(c_.user))
      throw std::runtime_error("continuation hook refused the reset");
  }
  void BeforeRestore() override {
    if (c_.before_restore && c_.before_restore(c_.user))
      throw std::runtime_error("continuation hook refused the restore");
  }

private:
  lfm3_continuation_hooks c_;
};

struct lfm3_session {
  std::unique_ptr<lfm3::Session> session;
  std::unique_ptr<CHooks> hooks;
};

lfm3_model* lfm3_model_load(const lfm3_weights* host) {
  if (!host) {
    Fail(LFM3_ERR_INVALID, "no weights");
    return nullptr;
  }
  std::string error;
  auto m = lfm3::Model::Load(*host, &error);
  if (!m) {
    Fail(LFM3_ERR_INVALID, error);
    return nullptr;
  }
  return new lfm3_model{std::move(m)};
}
void lfm3_model_free(lfm3_model* model) { delete model; }
int lfm3_model_config(const lfm3_model* model, lfm3_config* out) {
  if (!model || !out)
    return Fail(LFM3_ERR_INVALID, "null argument");
  *out = model->model->config();
  return LFM3_OK;
}
size_t lfm3_model_weight_bytes(const lfm3_model* model) {
  return model ? model->model->weight_bytes() : 0;
}

lfm3_session* lfm3_session_create(lfm3_model* model, uint32_t context) {
  if (!model) {
    Fail(LFM3_ERR_INVALID, "no model");
    return nullptr;
  }
  std::string error;
  try {
    auto s = model->model->CreateSession(context, &error);
    if (!s) {
      Fail(LFM3_ERR_INVALID, error);
      return nullptr;
    }
    return new lfm3_session{std::move(s), nullptr};
  } catch (const std::exception& e) {
    Fail(LFM3_ERR_CUDA, e.what());
    return nullptr;
  }
}
void lfm3_session_free(lfm3_session* session) { delete session; }

static int SessionStatus(const lfm3::Session& s, const std::string& error) {
  if (error.find("device wait") != std::string::npos)
    return Fail(LFM3_ERR_DEVICE_WAIT, error);
  return Fail(s.IsCoherent() ? LFM3_ERR_INVALID : LFM3_ERR_POISONED, error);
}

int lfm3_session_forward(lfm3_session* session, const uint32_t* tokens,
                         size_t n, float* logits) {
  if (!session || (!tokens && n))
    return Fail(LFM3_ERR_INVALID, "null argument");
  auto& s = *session->session;
  std::string error;
  const std::span<float> out =
      logits ? std::span<float>(logits, s.config().vocab) : std::span<float>();
  if (!s.Forward(std::span<const uint32_t>(tokens, n), out, &error))
    return SessionStatus(s, error);
  return LFM3_OK;
}

int lfm3_session_forward_batch(lfm3_session* const* sessions,
                               const uint32_t* tokens, size_t count,
                               float* const* logits) {
  if (!sessions || !tokens || !count || count > lfm3::kMaxBatch)
    return Fail(LFM3_ERR_INVALID, "batch must hold 1..8 sessions");
  lfm3::Session* batch[lfm3::kMaxBatch];
  std::span<float> outs[lfm3::kMaxBatch];
  for (size_t r = 0; r < count; ++r) {
    if (!sessions[r])
      return Fail(LFM3_ERR_INVALID, "null session");
    batch[r] = sessions[r]->session.get();
    const size_t vocab = batch[r]->config().vocab;
    outs[r] = logits && logits[r] ? std::span<float>(logits[r], vocab)
                                  : std::span<float>();
  }
  std::string error;
  if (!lfm3::Session::ForwardBatch(
          std::span<lfm3::Session* const>(batch, count),
          std::span<const uint32_t>(tokens, count),
          logits ? std::span<const std::span<float>>(outs, count)
                 : std::span<const std::span<float>>(),
          &error)) {
    bool poisoned = false;
    for (size_t r = 0; r < count; ++r)
      poisoned = poisoned || !batch[r]->IsCoherent();
    if (error.find("device wait") != std::string::npos)
      return Fail(LFM3_ERR_DEVICE_WAIT, error);
    return Fail(poisoned ? LFM3_ERR_POISONED : LFM3_ERR_INVALID, error);
  }
  return LFM3_OK;
}

int lfm3_session_forward_batch_sample(lfm3_session* const* sessions,
                                      const uint32_t* tokens, size_t count,
                                      const lfm3_sampler* sampler,
                                      const uint32_t* recent,
                                      const uint32_t* recent_count,
                                      const uint64_t* seeds, uint32_t* next) {
  if (!sessions || !tokens || !count || count > lfm3::kMaxBatch || !next)
    return Fail(LFM3_ERR_INVALID, "batch must hold 1..8 sessions");
  lfm3::Session* batch[lfm3::kMaxBatch];
  for (size_t r = 0; r < count; ++r) {
    if (!sessions[r])
      return Fail(LFM3_ERR_INVALID, "null session");
    batch[r] = sessions[r]->session.get();
  }
  lfm3::SampleControls c{};
  if (const int e = SampleArgs(sampler, int(count),
                               int(batch[0]->config().vocab), recent,
                               recent_count, seeds, &c))
    return e;
  std::string error;
  if (!lfm3::Session::ForwardBatchSample(
          std::span<lfm3::Session* const>(batch, count),
          std::span<const uint32_t>(tokens, count), c, recent, recent_count,
          seeds, std::span<uint32_t>(next, count), &error)) {
    bool poisoned = false;
    for (size_t r = 0; r < count; ++r)
      poisoned = poisoned || !batch[r]->IsCoherent();
    if (error.find("device wait") != std::string::npos)
      return Fail(LFM3_ERR_DEVICE_WAIT, error);
    return Fail(poisoned ? LFM3_ERR_POISONED : LFM3_ERR_INVALID, error);
  }
  return LFM3_OK;
}

int lfm3_session_forward_batch_inputs(lfm3_session* const* sessions,
                                      const uint32_t* tokens,
                                      const float* const* rows, size_t count,
                                      int logits) {
  if (!sessions || !tokens || !count || count > lfm3::kMaxBatch)
    return Fail(LFM3_ERR_INVALID, "batch must hold 1..8 sessions");
  lfm3::Session* batch[lfm3::kMaxBatch];
  for (size_t r = 0; r < count; ++r) {
    if (!sessions[r])
      return Fail(LFM3_ERR_INVALID, "null session");
    batch[r] = sessions[r]->session.get();
  }
  std::string error;
  if (!lfm3::Session::ForwardBatchInputs(
          std::span<lfm3::Session* const>(batch, count),
          std::span<const uint32_t>(tokens, count),
          rows ? std::span<const float* const>(rows, count)
               : std::span<const float* const>(),
          logits != 0, &error)) {
    bool poisoned = false;
    for (size_t r = 0; r < count; ++r)
      poisoned = poisoned || !batch[r]->IsCoherent();
    if (error.find("device wait") != std::string::npos)
      return Fail(LFM3_ERR_DEVICE_WAIT, error);
    return Fail(poisoned ? LFM3_ERR_POISONED : LFM3_ERR_INVALID, error);
  }
  return LFM3_OK;
}

int lfm3_session_forward_embeddings(lfm3_session* session, const float* rows,
                                    size_t n, int on_device, float* logits) {
  if (!session || !rows || !n)
    return Fail(LFM3_ERR_INVALID, "null argument");
  auto& s = *session->session;
  const auto& c = s.config();
  std::string error;
  if (!s.ForwardEmbeddings(
          std::span<const float>(rows, n * c.hidden), on_device != 0,
          logits ? std::span<float>(logits, c.vocab) : std::span<float>(),
          &error))
    return SessionStatus(s, error);
  return LFM3_OK;
}

int lfm3_session_forward_inputs(lfm3_session* session,
                                const lfm3_input* inputs, size_t count,
                                float* logits) {
  if (!session || (!inputs && count))
    return Fail(LFM3_ERR_INVALID, "null argument");
  auto& s = *session->session;
  const auto& c = s.config();
  std::vector<lfm3::Session::Input> runs(count);
  for (size_t i = 0; i < count; ++i) {
    const lfm3_input& in = inputs[i];
    if ((in.n_tokens && !in.tokens) || (in.n_rows && !in.rows))
      return Fail(LFM3_ERR_INVALID, "null input run");
    runs[i].tokens = std::span<const uint32_t>(in.tokens, in.n_tokens);
    runs[i].rows = std::span<const float>(in.rows, in.n_rows * c.hidden);
  }
  std::string error;
  if (!s.ForwardInputs(
          runs, logits ? std::span<float>(logits, c.vocab) : std::span<float>(),
          &error))
    return SessionStatus(s, error);
  return LFM3_OK;
}

int lfm3_session_speculate(lfm3_session* session, uint32_t token) {
  if (!session)
    return Fail(LFM3_ERR_INVALID, "null session");
  session->session->Speculate(token);
  return LFM3_OK;
}

int lfm3_session_forward_decision(lfm3_session* session,
                                  const uint32_t* tokens, size_t n,
                                  float* logits) {
  (void)tokens;
  (void)n;
  (void)logits;
  if (!session)
    return Fail(LFM3_ERR_INVALID, "null session");
  return Fail(LFM3_ERR_UNSUPPORTED,
              "d1 decision passes (bidirectional attention) are not built");
}

int lfm3_session_set_continuation_hooks(lfm3_session* session,
                                        const lfm3_continuation_hooks* hooks) {
  if (!session)
    return Fail(LFM3_ERR_INVALID, "null session");
  session->session->SetContinuationHooks(nullptr);
  session->hooks = hooks ? std::make_unique<CHooks>(*hooks) : nullptr;
  session->session->SetContinuationHooks(session->hooks.get());
  return LFM3_OK;
}

int lfm3_session_prepare_logits(lfm3_session* session) {
  if (!session)
    return Fail(LFM3_ERR_INVALID, "null session");
  std::string error;
  if (!session->session->PrepareLogits(&error))
    return SessionStatus(*session->session, error);
  return LFM3_OK;
}

int lfm3_session_begin_restore(lfm3_session* session) {
  if (!session)
    return Fail(LFM3_ERR_INVALID, "null session");
  std::string error;
  if (!session->session->BeginRestore(&error))
    return Fail(LFM3_ERR_CUDA, error);
  return LFM3_OK;
}

int lfm3_session_finish_restore(lfm3_session* session, uint32_t position) {
  if (!session)
    return Fail(LFM3_ERR_INVALID, "null session");
  std::string error;
  if (!session->session->FinishRestore(position, &error))
    return Fail(LFM3_ERR_INVALID, error);
  return LFM3_OK;
}

int lfm3_session_read_logits(lfm3_session* session, float* logits) {
  if (!session || !logits)
    return Fail(LFM3_ERR_INVALID, "null argument");
  auto& s = *session->session;
  std::string error;
  if (!s.ReadLogits(std::span<float>(logits, s.config().vocab), &error))
    return SessionStatus(s, error);
  return LFM3_OK;
}

int lfm3_session_read_hidden(lfm3_session* session, float* hidden) {
  if (!session || !hidden)
    return Fail(LFM3_ERR_INVALID, "null argument");
  auto& s = *session->session;
  std::string error;
  if (!s.ReadHidden(std::span<float>(hidden, s.config().hidden), &error))
    return SessionStatus(s, error);
  return LFM3_OK;
}

int lfm3_session_reset(lfm3_session* session) {
  if (!session)
    return Fail(LFM3_ERR_INVALID, "null argument");
  std::string error;
  if (!session->session->Reset(&error))
    return Fail(LFM3_ERR_CUDA, error);
  return LFM3_OK;
}

uint32_t lfm3_session_position(const lfm3_session* session) {
  return session ? session->session->Position() : 0;
}
int lfm3_session_is_coherent(const lfm3_session* session) {
  return session && session->session->IsCoherent() ? 1 : 0;
}
void* lfm3_session_stream(const lfm3_session* session) {
  return session ? session->session->DeviceStream() : nullptr;
}
void* lfm3_session_continuation_data(const lfm3_session* session, int tensor,
                                     size_t layer) {
  if (!session || tensor < 0 || tensor > 4)
    return nullptr;
  return session->session->ContinuationData(
      static_cast<lfm3::ContinuationTensor>(tensor), layer);
}
uint32_t lfm3_session_ring_capacity(const lfm3_session* session,
                                    size_t layer) {
  return session ? session->session->RingCapacity(layer) : 0;
}
struct lfm3_scheduler {
  std::unique_ptr<lfm3::Scheduler> scheduler;
};

lfm3_scheduler* lfm3_scheduler_create(lfm3_model* model,
                                      const lfm3_sampler* sampler) {
  if (!model || !sampler) {
    Fail(LFM3_ERR_INVALID, "null argument");
    return nullptr;
  }
  lfm3::SampleControls c{};
  if (const char* why = lfm3::sample_controls(
          sampler->temperature, sampler->top_k, sampler->repeat_penalty,
          int(model->model->config().vocab), &c)) {
    Fail(LFM3_ERR_INVALID, why);
    return nullptr;
  }
  try {
    auto* s = new lfm3_scheduler;
    s->scheduler = std::make_unique<lfm3::Scheduler>(model->model, c);
    return s;
  } catch (const std::exception& e) {
    Fail(LFM3_ERR_CUDA, e.what());
    return nullptr;
  }
}
void lfm3_scheduler_free(lfm3_scheduler* scheduler) { delete scheduler; }
int lfm3_scheduler_admit(lfm3_scheduler* scheduler, const uint32_t* prompt,
                         size_t n, uint32_t max_new, uint64_t seed,
                         uint32_t context) {
  if (!scheduler || (!prompt && n))
    return Fail(LFM3_ERR_INVALID, "null argument");
  std::string error;
  try {
    const int id = scheduler->scheduler->Admit(
        std::span<const uint32_t>(prompt, n), max_new, seed, context, &error);
    return id >= 0 ? id : Fail(LFM3_ERR_INVALID, error);
  } catch (const std::exception& e) {
    return Fail(LFM3_ERR_CUDA, e.what());
  }
}
int lfm3_scheduler_step(lfm3_scheduler* scheduler, lfm3_step_stats* stats) {
  if (!scheduler)
    return Fail(LFM3_ERR_INVALID, "null argument");
  lfm3::Scheduler::StepStats st;
  std::string error;
  const bool ok = scheduler->scheduler->Step(&st, &error);
  if (stats)
    *stats = lfm3_step_stats{st.pass_request, st.pass_rows, st.round_rows,
                             st.finished, st.pass_ms, st.round_ms};
  if (ok)
    return LFM3_OK;
  return Fail(error.find("device wait") != std::string::npos
                  ? LFM3_ERR_DEVICE_WAIT
                  : LFM3_ERR_CUDA,
              error);
}
int lfm3_scheduler_idle(const lfm3_scheduler* scheduler) {
  return scheduler && scheduler->scheduler->Idle() ? 1 : 0;
}
size_t lfm3_scheduler_tokens(const lfm3_scheduler* scheduler, int id,
                             uint32_t* out, size_t cap) {
  if (!scheduler)
    return 0;
  const auto t = scheduler->scheduler->Tokens(id);
  if (out)
    std::copy(t.begin(), t.begin() + std::min(cap, t.size()), out);
  return t.size();
}
int lfm3_scheduler_finished(const lfm3_scheduler* scheduler, int id) {
  if (!scheduler || !scheduler->scheduler->Finished(id))
    return 0;
  return scheduler->scheduler->Failed(id) ? 2 : 1;
}

uint32_t lfm3_snapshot_signature(const lfm3_config* config) {
  return config ? lfm3::SnapshotSignature(*config) : 0;
}
size_t lfm3_session_snapshot_bytes(const lfm3_session* session) {
  return session ? session->session->SnapshotBytes() : 0;
}
int lfm3_session_save_snapshot(lfm3_session* session, uint8_t* out,
                               size_t bytes) {
  if (!session || !out)
    return Fail(LFM3_ERR_INVALID, "null argument");
  if (!session->session->IsCoherent())
    return Fail(LFM3_ERR_POISONED, "cannot snapshot a poisoned LFM3 session");
  try {
    const auto data = session->session->SaveSnapshot();
    if (data.size() != bytes)
      return Fail(LFM3_ERR_INVALID, "snapshot buffer size mismatch");
    std::memcpy(out, data.data(), bytes);
    return LFM3_OK;
  } catch (const std::exception& e) {
    return Fail(LFM3_ERR_CUDA, e.what());
  }
}
int lfm3_session_restore_snapshot(lfm3_session* session, const uint8_t* data,
                                  size_t bytes) {
  if (!session || (!data && bytes))
    return Fail(LFM3_ERR_INVALID, "null argument");
  std::string error;
  if (!session->session->RestoreSnapshot(
          std::span<const uint8_t>(data, bytes), &error))
    return SessionStatus(*session->session, error);
  return LFM3_OK;
}
int lfm3_session_set_profiling(lfm3_session* session, int on) {
  if (!session)
    return Fail(LFM3_ERR_INVALID, "null argument");
  session->session->SetProfiling(on != 0);
  return LFM3_OK;
}
int lfm3_session_take_profile(lfm3_session* session, double* ms,
                              long long* launches) {
  if (!session)
    return Fail(LFM3_ERR_INVALID, "null argument");
  session->session->TakeProfile(ms, launches);
  return LFM3_OK;
}
unsigned long long lfm3_cuda_launch_count(void) { return lfm3::launch_count(); }

int lfm3_session_inject_failure(lfm3_session* session, int after_calls) {
  if (!session || after_calls < 0)
    return Fail(LFM3_ERR_INVALID, "invalid failure injection");
  session->session->InjectFailure(after_calls);
  return LFM3_OK;
}

}  // extern "C"
