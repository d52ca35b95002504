// The reference's engine header (engine.hpp) compiled with this library's
// definitions (include/lfm3_engine.inl), and linked with the reference's
// weights.cpp / config.cpp and liblfm3_cuda.so. main() takes the address of
// every public member the header declares, so the link fails if one has no
// definition of exactly its signature; then it runs the members that need
// no GPU and no GGUF file. TEST INFRASTRUCTURE (tests/test_ops_shim.py).
#include "engine.hpp"
#include "continuation_hooks.hpp"
#include "lfm3_engine.inl"

#include <cstdio>

namespace lfm = gufo::models::lfm3;

// Stand-ins for Gufo core's file mapping and the tokenizer's GGUF parser,
// which this check does not exercise.
std::unique_ptr<gufo::core::GgufReader> gufo::core::GgufReader::OpenFile(
    const std::string& path, std::string* error) {
  if (error)
    *error = "no such GGUF file: " + path;
  return nullptr;
}
std::unique_ptr<lfm::Tokenizer> lfm::Tokenizer::Load(const core::GgufReader&,
                                                     std::string* error) {
  if (error)
    *error = "no tokenizer";
  return nullptr;
}

int main() {
  using S = lfm::Session;
  using M = lfm::Model;
  using Decision1 = bool (S::*)(std::span<const std::uint32_t>,
                                std::span<const float>, std::span<float>,
                                std::string*);
  using Decision2 = bool (S::*)(std::span<const std::uint32_t>,
                                std::span<const float>,
                                std::span<const std::int32_t>,
                                std::span<const std::uint32_t>,
                                std::span<const std::uint32_t>,
                                std::span<float>, std::string*);
  // members as pointers (a missing definition fails the link)
  volatile bool taken[] = {
      &M::Load != nullptr, &M::CreateSession != nullptr,
      &M::config != nullptr, &M::tokenizer != nullptr, &M::OnNpu != nullptr,
      static_cast<Decision1>(&S::ForwardDecision) != nullptr,
      static_cast<Decision2>(&S::ForwardDecision) != nullptr,
      &S::ForwardDecisions != nullptr, &S::Speculate != nullptr,
      &S::Forward != nullptr, &S::ForwardBatch != nullptr,
      &S::ForwardBatchInputs != nullptr, &S::ForwardEmbeddings != nullptr,
      &S::ForwardInputs != nullptr, &S::ReadHidden != nullptr,
      &S::DeviceHidden != nullptr, &S::DeviceStream != nullptr,
      &S::Reset != nullptr, &S::Position != nullptr,
      &S::SnapshotBytes != nullptr, &S::SaveSnapshot != nullptr,
      &S::RestoreSnapshot != nullptr, &S::ReadLogits != nullptr,
      &S::SetContinuationHooks != nullptr, &S::ContinuationData != nullptr,
      &S::RingCapacity != nullptr, &S::IsCoherent != nullptr,
      &S::PrepareLogits != nullptr, &S::BeginRestore != nullptr,
      &S::FinishRestore != nullptr};
  int failures = 0;
  const auto expect = [&](bool ok, const char* what) {
    if (!ok) {
      std::printf("FAIL %s\n", what);
      ++failures;
    }
  };
  std::string error;
  expect(!M::Load("/nonexistent.gguf", &error) &&
             error.find("no such GGUF file") != std::string::npos,
         "Load reports the reader's error");
  error.clear();
  expect(!M::Load("/nonexistent.gguf", &error, 0, "bundle") &&
             error.find("NPU") != std::string::npos,
         "Load refuses the NPU backbone");
  // the bound weights' description: a d1 model is refused, a text model's
  // geometry and tensors carry over
  lfm::Weights w;
  w.config.hidden = 2048;
  w.config.vocab = 65536;
  w.config.layers = {lfm::LayerType::kConvolution,
                     lfm::LayerType::kSlidingAttention};
  w.config.kv_heads = {0, 8};
  w.layers.resize(2);
  w.layers[1].q = {reinterpret_cast<const void*>(0x1000),
                   gufo::core::GgmlType::kQ8_0, 2048, 2048, 2048 * 2176};
  auto d = std::make_unique<lfm3_weights>();
  expect(lfm::lfm3_cuda_detail::Describe(w, d.get(), &error) &&
             d->config.n_layers == 2 && d->config.hidden == 2048 &&
             d->config.layer_type[1] == LFM3_SLIDING_ATTENTION &&
             d->config.kv_heads[1] == 8 && d->layers[1].q.type == LFM3_Q8_0 &&
             d->layers[1].q.bytes == 2048u * 2176u,
         "Describe");
  w.config.decision = true;
  expect(!lfm::lfm3_cuda_detail::Describe(w, d.get(), &error),
         "Describe refuses d1 models");
  std::printf("members %zu failures %d\n", sizeof(taken) / sizeof(taken[0]),
              failures);
  return failures;
}
