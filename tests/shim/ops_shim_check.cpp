// The reference's operator header (hip/ops.hpp) compiled with this
// library's definitions (include/lfm3_gpu_ops.inl). main() takes the
// address of every function the header declares, so linking against
// liblfm3_cuda.so fails if a declaration has no definition of exactly its
// signature; then it runs the functions that need no GPU. TEST
// INFRASTRUCTURE (tests/test_ops_shim.py).
#include "hip/ops.hpp"
#include "lfm3_gpu_ops.inl"

#include <cstdio>
#include <stdexcept>

namespace gpu = gufo::models::lfm3::gpu;
using gufo::models::lfm3::Tensor;

int main() {
  using BiHalf = void (*)(const float*, const gpu::Half*, const gpu::Half*,
                          const float*, float*, int, int, int, hipStream_t,
                          const std::int32_t*, int);
  using BiFloat = void (*)(const float*, const float*, const float*, float*,
                           int, int, int, int, hipStream_t);
  const void* declared[] = {
      reinterpret_cast<const void*>(&gpu::Embed),
      reinterpret_cast<const void*>(&gpu::DenseWorkspaceBytes),
      reinterpret_cast<const void*>(&gpu::SplitPartialBytes),
      reinterpret_cast<const void*>(&gpu::SharesSplit),
      reinterpret_cast<const void*>(&gpu::Project),
      reinterpret_cast<const void*>(&gpu::ProjectSwiGLU),
      reinterpret_cast<const void*>(&gpu::ProjectFfn),
      reinterpret_cast<const void*>(&gpu::ResidualNorm),
      reinterpret_cast<const void*>(&gpu::Dense),
      reinterpret_cast<const void*>(&gpu::ShortConv),
      reinterpret_cast<const void*>(&gpu::RopeFrequencies),
      reinterpret_cast<const void*>(&gpu::Rope),
      reinterpret_cast<const void*>(&gpu::Attention),
      reinterpret_cast<const void*>(&gpu::AttentionScratchBytes),
      reinterpret_cast<const void*>(static_cast<BiHalf>(&gpu::BidirectionalAttention)),
      reinterpret_cast<const void*>(static_cast<BiFloat>(&gpu::BidirectionalAttention)),
      reinterpret_cast<const void*>(&gpu::SupportsBidirectionalAttention),
      reinterpret_cast<const void*>(&gpu::SelectRows),
      reinterpret_cast<const void*>(&gpu::PackKV),
      reinterpret_cast<const void*>(&gpu::StoreKV),
      reinterpret_cast<const void*>(&gpu::PromptHeads),
      reinterpret_cast<const void*>(&gpu::DecodeHeads),
      reinterpret_cast<const void*>(&gpu::LaunchBatchedRMSNorm),
      reinterpret_cast<const void*>(&gpu::LaunchBatchedPerHeadRMSNorm),
      reinterpret_cast<const void*>(&gpu::LaunchBatchedResidualAdd),
      reinterpret_cast<const void*>(&gpu::LaunchBatchedSwiGLUActivation),
      reinterpret_cast<const void*>(&gpu::LaunchGEMV),
      reinterpret_cast<const void*>(&gpu::LaunchBatchedQuantGEMMFp32),
      reinterpret_cast<const void*>(&gpu::LaunchExactBf16GEMMFp32SmallBatch),
  };
  int missing = 0;
  for (const void* f : declared)
    missing += f == nullptr;

  // host-only behaviour (no device memory is touched)
  int failures = 0;
  const auto expect = [&](bool ok, const char* what) {
    if (!ok) {
      std::printf("FAIL %s\n", what);
      ++failures;
    }
  };
  expect(gpu::DenseWorkspaceBytes(16, 2048) > 0, "DenseWorkspaceBytes");
  expect(gpu::SplitPartialBytes() > 0, "SplitPartialBytes");
  expect(!gpu::SupportsBidirectionalAttention(16, 4, 128),
         "SupportsBidirectionalAttention");
  // payload pointers are never dereferenced on the host
  Tensor q8{reinterpret_cast<const void*>(0x10000),
            gufo::core::GgmlType::kQ8_0, 2048, 512, 512 * 2176};
  Tensor bf{reinterpret_cast<const void*>(0x20000),
            gufo::core::GgmlType::kBF16, 2048, 512, 512 * 4096};
  float* out = nullptr;
  const gpu::Output both[] = {{&q8, out}, {&q8, out}};
  const gpu::Output mixed[] = {{&q8, out}, {&bf, out}};
  gpu::DenseWorkspace ws{reinterpret_cast<void*>(0x30000)};
  expect(gpu::SharesSplit(both, gpu::kPromptRows, ws), "SharesSplit prompt");
  expect(!gpu::SharesSplit(both, gpu::kPromptRows - 1, ws),
         "SharesSplit decode rows");
  expect(!gpu::SharesSplit(mixed, 64, ws), "SharesSplit mixed types");
  expect(!gpu::SharesSplit(both, 64, {}), "SharesSplit without workspace");
  bool threw = false;
  try {
    gpu::BidirectionalAttention(nullptr, static_cast<const gpu::Half*>(nullptr),
                                nullptr, nullptr, nullptr, 1, 16, 4, nullptr);
  } catch (const std::invalid_argument&) {
    threw = true;
  }
  expect(threw, "BidirectionalAttention refuses");
  std::printf("declared %zu missing %d failures %d\n",
              sizeof(declared) / sizeof(declared[0]), missing, failures);
  return missing || failures;
}
