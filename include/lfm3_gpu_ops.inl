// Definitions of the reference's operator functions
// (namespace gufo::models::lfm3::gpu, hip/ops.hpp:12-151) over this
// library's C ABI (lfm3_cuda.h): the drop-in for hip/ops.hip and
// hip/q8_prefill.hpp.
//
// Use: in exactly one translation unit of the extension, include the
// reference's hip/ops.hpp, then this file, and link liblfm3_cuda.so. The
// build supplies a <hip/hip_runtime.h> that maps the stream type,
//     #include <cuda_runtime.h>
//     using hipStream_t = cudaStream_t;
// so ops.hpp's declarations keep their names and argument meaning with CUDA
// streams. Errors follow the reference: shapes this build does not run throw
// std::invalid_argument (hip/ops.hip:2293-2294), ResidualNorm returns false
// for widths it does not run, CUDA failures throw std::runtime_error.
//
// Not built (they serve the d1 decision passes and the vision and audio
// encoders): BidirectionalAttention (both overloads) and
// LaunchBatchedPerHeadRMSNorm and LaunchBatchedSwiGLUActivation throw
// std::invalid_argument; SupportsBidirectionalAttention returns false.
#include <cstddef>
#include <cstdint>
#include <span>
#include <stdexcept>
#include <string>

#include "lfm3_cuda.h"

namespace gufo::models::lfm3::gpu {
namespace lfm3_cuda_detail {

inline lfm3_tensor T(const Tensor& t) {
  return {t.data, static_cast<std::uint32_t>(t.type), t.cols, t.rows,
          t.bytes};
}
inline lfm3_dense_workspace W(const DenseWorkspace& w) {
  return {w.quantized, w.row_max, w.partial, w.tickets};
}
inline void Check(int rc) {
  if (rc == LFM3_OK)
    return;
  if (rc == LFM3_ERR_INVALID || rc == LFM3_ERR_UNSUPPORTED)
    throw std::invalid_argument(lfm3_last_error());
  throw std::runtime_error(lfm3_last_error());
}
[[noreturn]] inline void NotBuilt(const char* what) {
  throw std::invalid_argument(std::string(what) +
                              " is not built for the B200 backbone");
}
// Output spans as the C ABI's descriptors (at most four outputs).
struct Outputs {
  lfm3_tensor tensors[4];
  lfm3_output outputs[4];
  int count = 0;
  explicit Outputs(std::span<const Output> in) {
    if (in.size() > 4)
      throw std::invalid_argument("at most four projections share an input");
    for (const Output& o : in) {
      tensors[count] = T(*o.weight);
      outputs[count] = {&tensors[count], o.out};
      ++count;
    }
  }
};

}  // namespace lfm3_cuda_detail

void Embed(const Tensor& weight, const std::uint32_t* tokens, float* out, int n,
           hipStream_t stream) {
  const lfm3_tensor w = lfm3_cuda_detail::T(weight);
  lfm3_cuda_detail::Check(lfm3_cuda_embed(&w, tokens, out, n, stream));
}

std::size_t DenseWorkspaceBytes(std::size_t rows, std::size_t K) {
  return lfm3_cuda_dense_workspace_bytes(rows, K);
}

std::size_t SplitPartialBytes() { return lfm3_cuda_split_partial_bytes(); }

bool SharesSplit(std::span<const Output> outputs, int n,
                 DenseWorkspace workspace) {
  if (outputs.empty() || outputs.size() > 4)
    return false;
  const lfm3_cuda_detail::Outputs o(outputs);
  const lfm3_dense_workspace ws = lfm3_cuda_detail::W(workspace);
  return lfm3_cuda_shares_split(o.outputs, o.count, n, &ws) != 0;
}

void Project(std::span<const Output> outputs, const float* x, int n,
             hipStream_t stream, DenseWorkspace workspace, bool split_ready) {
  const lfm3_cuda_detail::Outputs o(outputs);
  const lfm3_dense_workspace ws = lfm3_cuda_detail::W(workspace);
  lfm3_cuda_detail::Check(lfm3_cuda_project(o.outputs, o.count, x, n, stream,
                                            &ws, split_ready ? 1 : 0));
}

void ProjectSwiGLU(const Tensor& gate, const Tensor& up, const float* x,
                   float* out, float* up_scratch, int n, hipStream_t stream,
                   DenseWorkspace workspace, bool split_ready) {
  const lfm3_tensor g = lfm3_cuda_detail::T(gate), u = lfm3_cuda_detail::T(up);
  const lfm3_dense_workspace ws = lfm3_cuda_detail::W(workspace);
  lfm3_cuda_detail::Check(lfm3_cuda_project_swiglu(
      &g, &u, x, out, up_scratch, n, stream, &ws, split_ready ? 1 : 0));
}

void ProjectFfn(const Tensor& gate, const Tensor& up, const Tensor& down,
                const float* x, float* hidden, float* up_scratch, float* out,
                int n, hipStream_t stream, DenseWorkspace workspace,
                bool split_ready) {
  const lfm3_tensor g = lfm3_cuda_detail::T(gate), u = lfm3_cuda_detail::T(up),
                    d = lfm3_cuda_detail::T(down);
  const lfm3_dense_workspace ws = lfm3_cuda_detail::W(workspace);
  lfm3_cuda_detail::Check(lfm3_cuda_project_ffn(&g, &u, &d, x, hidden,
                                                up_scratch, out, n, stream,
                                                &ws, split_ready ? 1 : 0));
}

bool ResidualNorm(const float* branch, const Tensor* post_norm, float* x,
                  const Tensor* norm, float* z, int n, int hidden, float eps,
                  bool split, hipStream_t stream, DenseWorkspace workspace) {
  const lfm3_tensor p = post_norm ? lfm3_cuda_detail::T(*post_norm)
                                  : lfm3_tensor{},
                    q = norm ? lfm3_cuda_detail::T(*norm) : lfm3_tensor{};
  const lfm3_dense_workspace ws = lfm3_cuda_detail::W(workspace);
  const int rc = lfm3_cuda_residual_norm(
      branch, post_norm ? &p : nullptr, x, norm ? &q : nullptr, z, n, hidden,
      eps, split ? 1 : 0, stream, &ws);
  if (rc == LFM3_ERR_UNSUPPORTED)
    return false;  // the reference's "unsupported width" answer
  lfm3_cuda_detail::Check(rc);
  return true;
}

void Dense(const Tensor& weight, const float* x, float* out, int n,
           hipStream_t stream, DenseWorkspace workspace) {
  const lfm3_tensor w = lfm3_cuda_detail::T(weight);
  const lfm3_dense_workspace ws = lfm3_cuda_detail::W(workspace);
  lfm3_cuda_detail::Check(lfm3_cuda_dense(&w, x, out, n, stream, &ws));
}

void ShortConv(const float* projection, const float* weight, float* history,
               float* out, int n, int hidden, int width, hipStream_t stream,
               bool update) {
  lfm3_cuda_detail::Check(lfm3_cuda_short_conv(
      projection, weight, history, out, n, hidden, width, stream, update));
}

void RopeFrequencies(float* out, int dim, float theta, hipStream_t stream) {
  lfm3_cuda_detail::Check(lfm3_cuda_rope_frequencies(out, dim, theta, stream));
}

void Rope(float* x, const float* frequencies, const float* factors, int n,
          int heads, int dim, int position, hipStream_t stream) {
  lfm3_cuda_detail::Check(lfm3_cuda_rope(x, frequencies, factors, n, heads,
                                         dim, position, stream));
}

void Attention(const float* q, const Half* k, const Half* v, const float* gate,
               const Half* cache_k, const Half* cache_v, float* out, int n,
               int heads, int kv_heads, int dim, int position, int capacity,
               int window, hipStream_t stream, float* scratch) {
  lfm3_cuda_detail::Check(lfm3_cuda_attention(
      q, k, v, gate, cache_k, cache_v, out, n, heads, kv_heads, dim, position,
      capacity, window, stream, scratch));
}

std::size_t AttentionScratchBytes(int heads, int dim, int context, int rows) {
  return lfm3_cuda_attention_scratch_bytes(heads, dim, context, rows);
}

void BidirectionalAttention(const float*, const Half*, const Half*,
                            const float*, float*, int, int, int, hipStream_t,
                            const std::int32_t*, int) {
  lfm3_cuda_detail::NotBuilt("BidirectionalAttention");
}

void BidirectionalAttention(const float*, const float*, const float*, float*,
                            int, int, int, int, hipStream_t) {
  lfm3_cuda_detail::NotBuilt("BidirectionalAttention");
}

bool SupportsBidirectionalAttention(int, int, int) { return false; }

void SelectRows(const Tensor& source, const std::uint32_t* rows, void* out,
                int count, hipStream_t stream) {
  const lfm3_tensor s = lfm3_cuda_detail::T(source);
  lfm3_cuda_detail::Check(lfm3_cuda_select_rows(&s, rows, out, count, stream));
}

void PackKV(const float* k, const float* v, Half* k16, Half* v16,
            std::size_t count, hipStream_t stream) {
  lfm3_cuda_detail::Check(lfm3_cuda_pack_kv(k, v, k16, v16, count, stream));
}

void StoreKV(const Half* k, const Half* v, Half* cache_k, Half* cache_v, int n,
             int stride, int position, int capacity, hipStream_t stream) {
  lfm3_cuda_detail::Check(lfm3_cuda_store_kv(k, v, cache_k, cache_v, n, stride,
                                             position, capacity, stream));
}

void PromptHeads(float* q, float* k, const float* v, const float* q_norm,
                 const float* k_norm, const float* frequencies,
                 const float* factors, Half* k16, Half* v16, int n, int heads,
                 int kv_heads, int dim, int position, float eps,
                 hipStream_t stream) {
  lfm3_cuda_detail::Check(lfm3_cuda_prompt_heads(
      q, k, v, q_norm, k_norm, frequencies, factors, k16, v16, n, heads,
      kv_heads, dim, position, eps, stream));
}

void DecodeHeads(float* q, float* k, const float* v, const float* q_norm,
                 const float* k_norm, const float* frequencies,
                 const float* factors, Half* cache_k, Half* cache_v, int heads,
                 int kv_heads, int dim, int position, int capacity, float eps,
                 hipStream_t stream) {
  lfm3_cuda_detail::Check(lfm3_cuda_decode_heads(
      q, k, v, q_norm, k_norm, frequencies, factors, cache_k, cache_v, heads,
      kv_heads, dim, position, capacity, eps, stream));
}

void LaunchBatchedRMSNorm(const float* x, const float* weight, float* out,
                          void* out_bf16, std::size_t batch_size,
                          std::size_t dim, float eps, hipStream_t stream) {
  lfm3_cuda_detail::Check(lfm3_cuda_batched_rmsnorm(
      x, weight, out, out_bf16, batch_size, dim, eps, stream));
}

void LaunchBatchedPerHeadRMSNorm(const float*, const float*, float*,
                                 std::size_t, std::uint32_t, std::uint32_t,
                                 float, hipStream_t) {
  lfm3_cuda_detail::NotBuilt("LaunchBatchedPerHeadRMSNorm");
}

void LaunchBatchedResidualAdd(const float* a, const float* b, float* out,
                              std::size_t batch_size, std::size_t dim,
                              hipStream_t stream) {
  lfm3_cuda_detail::Check(
      lfm3_cuda_batched_residual_add(a, b, out, batch_size, dim, stream));
}

void LaunchBatchedSwiGLUActivation(const float*, const float*, float*, void*,
                                   std::size_t, hipStream_t) {
  lfm3_cuda_detail::NotBuilt("LaunchBatchedSwiGLUActivation");
}

void LaunchGEMV(const void* A, core::GgmlType a_type, const float* x, float* y,
                std::size_t M, std::size_t K, hipStream_t stream) {
  lfm3_cuda_detail::Check(lfm3_cuda_gemv(
      A, static_cast<std::uint32_t>(a_type), x, y, M, K, stream));
}

void LaunchBatchedQuantGEMMFp32(core::GgmlType type, const void* w,
                                const float* fp32_x, float* y,
                                std::size_t batch, std::size_t m, std::size_t k,
                                hipStream_t stream) {
  lfm3_cuda_detail::Check(lfm3_cuda_batched_quant_gemm_fp32(
      static_cast<std::uint32_t>(type), w, fp32_x, y, batch, m, k, stream));
}

void LaunchExactBf16GEMMFp32SmallBatch(const void* A, const float* X, float* Y,
                                       std::size_t batch_size, std::size_t M,
                                       std::size_t K, hipStream_t stream) {
  lfm3_cuda_detail::Check(lfm3_cuda_exact_bf16_gemm_fp32_small_batch(
      A, X, Y, batch_size, M, K, stream));
}

}  // namespace gufo::models::lfm3::gpu
