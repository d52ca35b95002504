// Definitions of the reference's engine classes (gufo::models::lfm3::Model
// and Session, engine.hpp:17-163) over this library's C ABI (lfm3_cuda.h):
// the drop-in for engine.cpp and upload.cpp on the B200.
//
// Use: in exactly one translation unit of the extension, include the
// reference's engine.hpp and continuation_hooks.hpp, then this file, and
// link liblfm3_cuda.so together with the extension's weights.cpp,
// config.cpp and tokenizer.cpp (Weights::Bind and Tokenizer::Load parse the
// GGUF file that Gufo core's GgufReader::OpenFile maps). Model::Load binds
// the weights exactly as the reference does and hands the bound host tensors
// to lfm3_model_load, which uploads them; every Session member forwards to
// the matching lfm3_session_* entry point, so runner.cpp and the
// continuation adapter compile and run unchanged.
//
// Not built: the NPU backbone (a non-empty npu_bundle makes Load fail) and
// the d1 decision passes (ForwardDecision / ForwardDecisions return false
// with an error); Speculate has nothing to start on the GPU.
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "lfm3_cuda.h"

namespace gufo::models::lfm3 {
namespace lfm3_cuda_detail {

inline lfm3_tensor Tensor_(const Tensor& t) {
  return {t.data, static_cast<std::uint32_t>(t.type), t.cols, t.rows,
          t.bytes};
}
inline bool Fail(std::string* error, const std::string& message) {
  if (error)
    *error = message;
  return false;
}
inline bool Status(int rc, std::string* error) {
  return rc == LFM3_OK || Fail(error, lfm3_last_error());
}
inline void Throw(int rc) {
  if (rc != LFM3_OK)
    throw std::runtime_error(lfm3_last_error());
}
// The bound host weights as the C ABI's descriptors.
inline bool Describe(const Weights& w, lfm3_weights* out, std::string* error) {
  const Config& c = w.config;
  if (c.decision)
    return Fail(error, "d1 decision models are not built for the B200 backbone");
  if (w.layers.size() > LFM3_MAX_LAYERS || c.layers.size() != w.layers.size() ||
      c.kv_heads.size() < w.layers.size())
    return Fail(error, "invalid LFM3 layer count");
  *out = lfm3_weights{};
  lfm3_config& d = out->config;
  d.hidden = c.hidden;
  d.intermediate = c.intermediate;
  d.vocab = c.vocab;
  d.context = c.context;
  d.heads = c.heads;
  d.head_dim = c.head_dim;
  d.window = c.window;
  d.conv_width = c.conv_width;
  d.n_layers = static_cast<std::uint32_t>(w.layers.size());
  d.eps = c.eps;
  d.theta = c.theta;
  d.theta_swa = c.theta_swa;
  for (std::size_t i = 0; i < w.layers.size(); ++i) {
    d.kv_heads[i] = c.kv_heads[i];
    // LayerType and lfm3_layer_type share their values (config.hpp:7)
    d.layer_type[i] = static_cast<std::uint32_t>(c.layers[i]);
    const LayerWeights& l = w.layers[i];
    lfm3_layer& o = out->layers[i];
    o.norm = Tensor_(l.norm);
    o.ffn_norm = Tensor_(l.ffn_norm);
    o.post_norm = Tensor_(l.post_norm);
    o.post_ffn_norm = Tensor_(l.post_ffn_norm);
    o.gate = Tensor_(l.gate);
    o.up = Tensor_(l.up);
    o.down = Tensor_(l.down);
    o.conv = Tensor_(l.conv);
    o.in_proj = Tensor_(l.in_proj);
    o.out_proj = Tensor_(l.out_proj);
    o.q = Tensor_(l.q);
    o.k = Tensor_(l.k);
    o.v = Tensor_(l.v);
    o.q_norm = Tensor_(l.q_norm);
    o.k_norm = Tensor_(l.k_norm);
    o.attn_gate = Tensor_(l.attn_gate);
    o.attn_out = Tensor_(l.attn_out);
  }
  out->embedding = Tensor_(w.embedding);
  out->output = Tensor_(w.output);
  out->output_norm = Tensor_(w.output_norm);
  out->rope_freqs = Tensor_(w.rope_freqs);
  return true;
}

}  // namespace lfm3_cuda_detail

struct Model::Impl {
  std::unique_ptr<core::GgufReader> reader;
  std::unique_ptr<Tokenizer> tokenizer;
  Weights weights;
  lfm3_model* model = nullptr;
  ~Impl() {
    if (model)
      lfm3_model_free(model);
  }
};

struct Session::Impl {
  std::shared_ptr<Model> model;  // outlives the session's device state
  lfm3_session* session = nullptr;
  ~Impl() {
    if (session)
      lfm3_session_free(session);
  }
};
struct Session::Npu {};

Model::Model() : impl_(std::make_unique<Impl>()) {}
Model::~Model() = default;

std::shared_ptr<Model> Model::Load(const std::string& path, std::string* error,
                                   std::uint32_t session_context,
                                   const std::string& npu_bundle) {
  (void)session_context;  // sessions allocate their state when created
  try {
    if (!npu_bundle.empty()) {
      lfm3_cuda_detail::Fail(error, "the NPU backbone is not built");
      return nullptr;
    }
    auto m = std::shared_ptr<Model>(new Model);
    m->impl_->reader = core::GgufReader::OpenFile(path, error);
    if (!m->impl_->reader)
      return nullptr;
    auto w = Weights::Bind(*m->impl_->reader, error);
    if (!w)
      return nullptr;
    m->impl_->weights = *w;
    auto described = std::make_unique<lfm3_weights>();
    if (!lfm3_cuda_detail::Describe(m->impl_->weights, described.get(), error))
      return nullptr;
    m->impl_->tokenizer = Tokenizer::Load(*m->impl_->reader, error);
    if (!m->impl_->tokenizer)
      return nullptr;
    m->impl_->model = lfm3_model_load(described.get());
    if (!m->impl_->model) {
      lfm3_cuda_detail::Fail(error, lfm3_last_error());
      return nullptr;
    }
    return m;
  } catch (const std::exception& e) {
    lfm3_cuda_detail::Fail(error, e.what());
    return nullptr;
  }
}

std::unique_ptr<Session> Model::CreateSession(std::uint32_t context,
                                              std::string* error) {
  try {
    if (!context || context > config().context)
      throw std::invalid_argument("invalid LFM3 context");
    auto session =
        std::unique_ptr<Session>(new Session(shared_from_this(), context));
    if (!session->impl_->session) {
      lfm3_cuda_detail::Fail(error, lfm3_last_error());
      return nullptr;
    }
    return session;
  } catch (const std::exception& e) {
    lfm3_cuda_detail::Fail(error, e.what());
    return nullptr;
  }
}

const Config& Model::config() const { return impl_->weights.config; }
const Tokenizer& Model::tokenizer() const { return *impl_->tokenizer; }
bool Model::OnNpu() const { return false; }

Session::Session(std::shared_ptr<Model> model, std::uint32_t context)
    : impl_(std::make_unique<Impl>()) {
  impl_->session = lfm3_session_create(model->impl_->model, context);
  impl_->model = std::move(model);
}
Session::~Session() = default;

bool Session::ForwardDecision(std::span<const std::uint32_t>,
                              std::span<const float>, std::span<float>,
                              std::string* error) {
  return lfm3_cuda_detail::Fail(error, "d1 decision passes are not built");
}
bool Session::ForwardDecision(std::span<const std::uint32_t>,
                              std::span<const float>,
                              std::span<const std::int32_t>,
                              std::span<const std::uint32_t>,
                              std::span<const std::uint32_t>, std::span<float>,
                              std::string* error) {
  return lfm3_cuda_detail::Fail(error, "d1 decision passes are not built");
}
bool Session::ForwardDecisions(std::span<const std::uint32_t>,
                               std::span<const float>,
                               std::span<const DecisionPrompt>,
                               std::span<const std::uint32_t>, std::span<float>,
                               std::string* error) {
  return lfm3_cuda_detail::Fail(error, "d1 decision passes are not built");
}

void Session::Speculate(std::uint32_t token) {
  (void)lfm3_session_speculate(impl_->session, token);
}

bool Session::Forward(std::span<const std::uint32_t> tokens,
                      std::span<float> logits, std::string* error) {
  return lfm3_cuda_detail::Status(
      lfm3_session_forward(impl_->session, tokens.data(), tokens.size(),
                           logits.empty() ? nullptr : logits.data()),
      error);
}

bool Session::ForwardBatch(std::span<Session* const> sessions,
                           std::span<const std::uint32_t> tokens,
                           std::span<std::span<float>> logits,
                           std::string* error) {
  if (sessions.empty() || sessions.size() > kMaxBatch ||
      tokens.size() != sessions.size() ||
      (!logits.empty() && logits.size() != sessions.size()))
    return lfm3_cuda_detail::Fail(error, "invalid LFM3 batch");
  lfm3_session* handles[kMaxBatch];
  float* outs[kMaxBatch];
  for (std::size_t r = 0; r < sessions.size(); ++r) {
    handles[r] = sessions[r] ? sessions[r]->impl_->session : nullptr;
    outs[r] = logits.empty() || logits[r].empty() ? nullptr : logits[r].data();
  }
  return lfm3_cuda_detail::Status(
      lfm3_session_forward_batch(handles, tokens.data(), sessions.size(),
                                 logits.empty() ? nullptr : outs),
      error);
}

bool Session::ForwardBatchInputs(std::span<Session* const> sessions,
                                 std::span<const std::uint32_t> tokens,
                                 std::span<const float* const> rows,
                                 bool logits, std::string* error) {
  if (sessions.empty() || sessions.size() > kMaxBatch ||
      tokens.size() != sessions.size() ||
      (!rows.empty() && rows.size() != sessions.size()))
    return lfm3_cuda_detail::Fail(error, "invalid LFM3 batch");
  lfm3_session* handles[kMaxBatch];
  for (std::size_t r = 0; r < sessions.size(); ++r)
    handles[r] = sessions[r] ? sessions[r]->impl_->session : nullptr;
  return lfm3_cuda_detail::Status(
      lfm3_session_forward_batch_inputs(handles, tokens.data(),
                                        rows.empty() ? nullptr : rows.data(),
                                        sessions.size(), logits ? 1 : 0),
      error);
}

bool Session::ForwardEmbeddings(std::span<const float> rows, bool on_device,
                                std::span<float> logits, std::string* error) {
  const std::size_t hidden = impl_->model->config().hidden;
  if (!hidden || rows.size() % hidden)
    return lfm3_cuda_detail::Fail(error, "invalid LFM3 embedding count");
  return lfm3_cuda_detail::Status(
      lfm3_session_forward_embeddings(
          impl_->session, rows.data(), rows.size() / hidden, on_device ? 1 : 0,
          logits.empty() ? nullptr : logits.data()),
      error);
}

bool Session::ForwardInputs(std::span<const Input> inputs,
                            std::span<float> logits, std::string* error) {
  const std::size_t hidden = impl_->model->config().hidden;
  std::vector<lfm3_input> runs(inputs.size());
  for (std::size_t i = 0; i < inputs.size(); ++i) {
    if (!hidden || inputs[i].rows.size() % hidden)
      return lfm3_cuda_detail::Fail(error, "invalid LFM3 embedding count");
    runs[i] = {inputs[i].tokens.data(), inputs[i].tokens.size(),
               inputs[i].rows.data(), inputs[i].rows.size() / hidden};
  }
  return lfm3_cuda_detail::Status(
      lfm3_session_forward_inputs(impl_->session, runs.data(), runs.size(),
                                  logits.empty() ? nullptr : logits.data()),
      error);
}

bool Session::ReadHidden(std::span<float> hidden, std::string* error) const {
  if (hidden.size() != impl_->model->config().hidden)
    return lfm3_cuda_detail::Fail(error, "hidden must hold hidden floats");
  return lfm3_cuda_detail::Status(
      lfm3_session_read_hidden(impl_->session, hidden.data()), error);
}

const float* Session::DeviceHidden() const {
  return static_cast<const float*>(lfm3_session_continuation_data(
      impl_->session, static_cast<int>(ContinuationTensor::kFrontier), 0));
}

void* Session::DeviceStream() const {
  return lfm3_session_stream(impl_->session);
}

bool Session::Reset(std::string* error) {
  return lfm3_cuda_detail::Status(lfm3_session_reset(impl_->session), error);
}

std::uint32_t Session::Position() const {
  return lfm3_session_position(impl_->session);
}

std::size_t Session::SnapshotBytes() const {
  return lfm3_session_snapshot_bytes(impl_->session);
}

std::vector<std::uint8_t> Session::SaveSnapshot() const {
  std::vector<std::uint8_t> out(SnapshotBytes());
  lfm3_cuda_detail::Throw(
      lfm3_session_save_snapshot(impl_->session, out.data(), out.size()));
  return out;
}

bool Session::RestoreSnapshot(std::span<const std::uint8_t> payload,
                              std::string* error) {
  return lfm3_cuda_detail::Status(
      lfm3_session_restore_snapshot(impl_->session, payload.data(),
                                    payload.size()),
      error);
}

bool Session::ReadLogits(std::span<float> logits, std::string* error) const {
  if (logits.size() != impl_->model->config().vocab)
    return lfm3_cuda_detail::Fail(error, "logits must hold vocab floats");
  return lfm3_cuda_detail::Status(
      lfm3_session_read_logits(impl_->session, logits.data()), error);
}

void Session::SetContinuationHooks(ContinuationHooks* hooks) {
  hooks_ = hooks;
  if (!hooks) {
    lfm3_cuda_detail::Throw(
        lfm3_session_set_continuation_hooks(impl_->session, nullptr));
    return;
  }
  // each callback refuses (nonzero) when the adapter's hook throws
  const lfm3_continuation_hooks c{
      hooks,
      [](void* user, std::uint32_t first, std::uint32_t end) {
        try {
          static_cast<ContinuationHooks*>(user)->BeforeWrite(first, end);
          return 0;
        } catch (...) {
          return 1;
        }
      },
      [](void* user) {
        try {
          static_cast<ContinuationHooks*>(user)->BeforeReset();
          return 0;
        } catch (...) {
          return 1;
        }
      },
      [](void* user) {
        try {
          static_cast<ContinuationHooks*>(user)->BeforeRestore();
          return 0;
        } catch (...) {
          return 1;
        }
      }};
  lfm3_cuda_detail::Throw(lfm3_session_set_continuation_hooks(impl_->session, &c));
}

void* Session::ContinuationData(ContinuationTensor tensor,
                                std::size_t layer) const {
  return lfm3_session_continuation_data(impl_->session,
                                        static_cast<int>(tensor), layer);
}

std::uint32_t Session::RingCapacity(std::size_t layer) const {
  return lfm3_session_ring_capacity(impl_->session, layer);
}

bool Session::IsCoherent() const {
  return lfm3_session_is_coherent(impl_->session) != 0;
}

void Session::PrepareLogits() {
  lfm3_cuda_detail::Throw(lfm3_session_prepare_logits(impl_->session));
}

void Session::BeginRestore() {
  lfm3_cuda_detail::Throw(lfm3_session_begin_restore(impl_->session));
}

void Session::FinishRestore(std::uint32_t position) {
  lfm3_cuda_detail::Throw(lfm3_session_finish_restore(impl_->session, position));
}

}  // namespace gufo::models::lfm3
