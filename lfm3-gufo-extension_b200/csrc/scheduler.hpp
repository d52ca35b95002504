// Continuous batching of independent sessions on one GPU: the step that the
// reference's host scheduler drives through its text runner. The runner's
// scheduling profile (runner.cpp:140-147) asks for prompt passes of at most
// 512 rows run in one layer group between decode rounds of at most 8
// sessions (runner.cpp:172-177); the runner's Prefill, AdvanceBatch and
// SelectNext (runner.cpp:249-351) become one Step here:
//   1. one prompt pass of at most 512 rows for the first admitted request
//      that has prompt rows left (first come, first served); after a
//      request's last pass its first token is selected on the device from
//      the pass's final row;
//   2. one decode round of up to 8 decoding requests (in admission order),
//      each advancing its pending token (Session::ForwardBatchSample), with
//      the next token selected on the device.
// A request decodes until it has selected max_new tokens. Every selection
// uses the scheduler's sampler over the request's last 64 tokens (its
// prompt's tail, then every token it has advanced) and a per-draw seed
// seed ^ (position * 0x9E3779B97F4A7C15), position = tokens advanced.
#pragma once
#include <cstdint>
#include <memory>
#include <span>
#include <string>
#include <vector>

#include "engine.hpp"

namespace lfm3 {

class Scheduler {
public:
  Scheduler(std::shared_ptr<Model> model, const SampleControls& controls);
  // Admits a request; returns its id, or -1 with *error (empty prompt, a
  // token outside the vocabulary, max_new of 0, a context below prompt +
  // max_new, or a session that cannot be created).
  int Admit(std::span<const uint32_t> prompt, uint32_t max_new, uint64_t seed,
            uint32_t context, std::string* error = nullptr);
  struct StepStats {
    int pass_request = -1;  // request of this step's prompt pass, or -1
    uint32_t pass_rows = 0;
    uint32_t round_rows = 0;  // requests the decode round advanced
    uint32_t finished = 0;    // requests completed by this step
    double pass_ms = 0, round_ms = 0;  // host time, results on the host
  };
  // One step. False with *error when a device call failed: the requests of
  // that call are retired (their sessions poisoned), the others go on.
  bool Step(StepStats* stats, std::string* error = nullptr);
  // No admitted request has work left.
  bool Idle() const;
  // The tokens a request has selected so far (empty for an unknown id).
  std::span<const uint32_t> Tokens(int id) const;
  bool Finished(int id) const;
  bool Failed(int id) const;

private:
  struct Request {
    std::unique_ptr<Session> session;
    std::vector<uint32_t> prompt;
    size_t done = 0;  // prompt rows advanced
    uint32_t max_new = 0;
    uint64_t seed = 0;
    std::vector<uint32_t> generated;
    uint32_t recent[kSampleMaxRecent] = {};  // ring of the last 64 tokens
    uint32_t recent_count = 0, recent_next = 0;
    bool failed = false;
    void Remember(uint32_t token);
    bool Decoding() const;
    bool Done() const;
  };
  static uint64_t DrawSeed(uint64_t seed, uint64_t position);
  std::shared_ptr<Model> model_;
  SampleControls controls_;
  std::vector<std::unique_ptr<Request>> requests_;
};

}  // namespace lfm3
