// C entry points around the reference's own CPU oracle — TEST INFRASTRUCTURE
// ONLY. Builds an in-memory GGUF view of an lfm3_weights description, binds
// it with the reference's Weights::Bind (weights.cpp:10-100, which validates
// it through Config::FromGguf, config.cpp:6-85) and drives
// Reference::Step (reference.cpp:72-168). Compiled with the reference's
// reference.cpp, weights.cpp and config.cpp, unmodified, by oracle/Makefile
// into oracle/_ref/libref_oracle.so.
#include <cstring>
#include <exception>
#include <memory>
#include <string>
#include <vector>

#include "../include/lfm3_types.h"
#include "reference.hpp"

namespace l = gufo::models::lfm3;
namespace core = gufo::core;
namespace {
struct Holder {
  core::GgufReader reader;
  l::Weights weights;
  std::unique_ptr<l::Reference> reference;
};
void AddTensor(core::GgufReader& r, const std::string& name,
               const lfm3_tensor& t, bool matrix) {
  if (!t.data)
    return;
  core::GgufTensorInfo info;
  info.dimensions = matrix ? std::vector<std::uint64_t>{t.cols, t.rows}
                           : std::vector<std::uint64_t>{t.cols};
  info.type = static_cast<core::GgmlType>(t.type);
  info.size_bytes = t.bytes;
  info.data = t.data;
  r.tensors[name] = info;
}
void Fill(core::GgufReader& r, const lfm3_weights& w) {
  const auto& c = w.config;
  auto u = [&](const char* key, std::uint64_t v) {
    r.metadata[std::string("lfm3.") + key].value = v;
  };
  auto f = [&](const char* key, float v) {
    r.metadata[std::string("lfm3.") + key].value = v;
  };
  r.metadata["general.architecture"].value = std::string("lfm3");
  u("block_count", c.n_layers);
  u("embedding_length", c.hidden);
  u("feed_forward_length", c.intermediate);
  u("context_length", c.context);
  u("attention.head_count", c.heads);
  u("attention.key_length", c.head_dim);
  u("attention.value_length", c.head_dim);
  u("rope.dimension_count", c.head_dim);
  u("attention.sliding_window", c.window);
  u("shortconv.l_cache", c.conv_width);
  f("attention.layer_norm_rms_epsilon", c.eps);
  f("rope.freq_base", c.theta);
  f("rope.freq_base_swa", c.theta_swa);
  r.metadata["tokenizer.ggml.tokens"].value =
      std::vector<std::string>(c.vocab);
  std::vector<std::uint64_t> kv, sw;
  for (std::uint32_t i = 0; i < c.n_layers; ++i) {
    kv.push_back(c.kv_heads[i]);
    sw.push_back(c.layer_type[i] == LFM3_SLIDING_ATTENTION ? 1 : 0);
  }
  r.metadata["lfm3.attention.head_count_kv"].value = kv;
  r.metadata["lfm3.attention.sliding_window_pattern"].value = sw;
  AddTensor(r, "token_embd.weight", w.embedding, true);
  if (w.output.data && w.output.data != w.embedding.data)
    AddTensor(r, "output.weight", w.output, true);
  AddTensor(r, "output_norm.weight", w.output_norm, false);
  AddTensor(r, "rope_freqs.weight", w.rope_freqs, false);
  for (std::uint32_t i = 0; i < c.n_layers; ++i) {
    const auto& L = w.layers[i];
    const auto p = "blk." + std::to_string(i) + ".";
    AddTensor(r, p + "attn_norm.weight", L.norm, false);
    AddTensor(r, p + "ffn_norm.weight", L.ffn_norm, false);
    AddTensor(r, p + "post_attention_norm.weight", L.post_norm, false);
    AddTensor(r, p + "post_ffw_norm.weight", L.post_ffn_norm, false);
    AddTensor(r, p + "ffn_gate.weight", L.gate, true);
    AddTensor(r, p + "ffn_up.weight", L.up, true);
    AddTensor(r, p + "ffn_down.weight", L.down, true);
    AddTensor(r, p + "shortconv.conv.weight", L.conv, true);
    AddTensor(r, p + "shortconv.in_proj.weight", L.in_proj, true);
    AddTensor(r, p + "shortconv.out_proj.weight", L.out_proj, true);
    AddTensor(r, p + "attn_q.weight", L.q, true);
    AddTensor(r, p + "attn_k.weight", L.k, true);
    AddTensor(r, p + "attn_v.weight", L.v, true);
    AddTensor(r, p + "attn_q_norm.weight", L.q_norm, false);
    AddTensor(r, p + "attn_k_norm.weight", L.k_norm, false);
    AddTensor(r, p + "attn_gate.weight", L.attn_gate, true);
    AddTensor(r, p + "attn_output.weight", L.attn_out, true);
  }
}
void Report(char* error, std::size_t bytes, const std::string& what) {
  if (error && bytes) {
    std::strncpy(error, what.c_str(), bytes - 1);
    error[bytes - 1] = 0;
  }
}
}  // namespace

extern "C" {
void* ref_oracle_create(const lfm3_weights* w, std::uint32_t context,
                        char* error, std::size_t error_bytes) {
  try {
    auto h = std::make_unique<Holder>();
    Fill(h->reader, *w);
    std::string message;
    auto bound = l::Weights::Bind(h->reader, &message);
    if (!bound) {
      Report(error, error_bytes, message);
      return nullptr;
    }
    h->weights = *bound;
    h->reference = std::make_unique<l::Reference>(h->weights, context);
    return h.release();
  } catch (const std::exception& e) {
    Report(error, error_bytes, e.what());
    return nullptr;
  }
}
int ref_oracle_step(void* handle, std::uint32_t token, float* logits) {
  auto* h = static_cast<Holder*>(handle);
  try {
    const auto vocab = h->weights.config.vocab;
    h->reference->Step(token, logits ? std::span<float>(logits, vocab)
                                     : std::span<float>());
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}
void ref_oracle_reset(void* handle) {
  static_cast<Holder*>(handle)->reference->Reset();
}
std::uint32_t ref_oracle_position(void* handle) {
  return static_cast<Holder*>(handle)->reference->Position();
}
void ref_oracle_destroy(void* handle) { delete static_cast<Holder*>(handle); }
}
