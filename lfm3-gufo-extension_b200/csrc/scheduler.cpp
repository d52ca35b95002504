// Continuous batching on one GPU; see scheduler.hpp.
#include "scheduler.hpp"

#include <chrono>

namespace lfm3 {

namespace {
double Ms(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(
             std::chrono::steady_clock::now() - t0)
      .count();
}
}  // namespace

void Scheduler::Request::Remember(uint32_t token) {
  recent[recent_next] = token;
  recent_next = (recent_next + 1) % kSampleMaxRecent;
  if (recent_count < uint32_t(kSampleMaxRecent))
    ++recent_count;
}

bool Scheduler::Request::Decoding() const {
  return !failed && done == prompt.size() && !generated.empty() &&
         generated.size() < max_new;
}

bool Scheduler::Request::Done() const {
  return failed || generated.size() >= max_new;
}

uint64_t Scheduler::DrawSeed(uint64_t seed, uint64_t position) {
  return seed ^ (position * 0x9E3779B97F4A7C15ull);
}

Scheduler::Scheduler(std::shared_ptr<Model> model,
                     const SampleControls& controls)
    : model_(std::move(model)), controls_(controls) {}

int Scheduler::Admit(std::span<const uint32_t> prompt, uint32_t max_new,
                     uint64_t seed, uint32_t context, std::string* error) {
  const auto fail = [&](const std::string& why) {
    if (error)
      *error = why;
    return -1;
  };
  if (prompt.empty() || max_new == 0)
    return fail("a request needs a prompt and at least one new token");
  for (const uint32_t t : prompt)
    if (t >= model_->config().vocab)
      return fail("prompt token outside the vocabulary");
  if (uint64_t(prompt.size()) + max_new > context)
    return fail("context below prompt + max_new");
  auto r = std::make_unique<Request>();
  r->session = model_->CreateSession(context, error);
  if (!r->session)
    return -1;
  r->prompt.assign(prompt.begin(), prompt.end());
  r->max_new = max_new;
  r->seed = seed;
  const size_t tail = std::min<size_t>(prompt.size(), kSampleMaxRecent);
  for (size_t i = prompt.size() - tail; i < prompt.size(); ++i)
    r->Remember(prompt[i]);
  r->generated.reserve(max_new);
  requests_.push_back(std::move(r));
  return int(requests_.size()) - 1;
}

bool Scheduler::Step(StepStats* stats, std::string* error) {
  StepStats local;
  StepStats& st = stats ? *stats : local;
  st = StepStats{};
  bool ok = true;
  const auto note = [&](const std::string& why) {
    if (error && ok)
      *error = why;
    ok = false;
  };
  // 1. one prompt pass, first come first served
  for (size_t id = 0; id < requests_.size(); ++id) {
    Request& r = *requests_[id];
    if (r.failed || r.done == r.prompt.size())
      continue;
    const auto t0 = std::chrono::steady_clock::now();
    const size_t n =
        std::min(Session::kPrefillChunk, r.prompt.size() - r.done);
    const std::span<const uint32_t> rows(r.prompt.data() + r.done, n);
    std::string why;
    bool pass_ok = r.session->Forward(rows, {}, &why);
    if (pass_ok) {
      r.done += n;
      st.pass_request = int(id);
      st.pass_rows = uint32_t(n);
      if (r.done == r.prompt.size()) {
        uint32_t token = 0;
        pass_ok = r.session->SampleLogits(
            controls_, r.recent, r.recent_count,
            DrawSeed(r.seed, r.session->Position()), &token, &why);
        if (pass_ok) {
          r.generated.push_back(token);
          if (r.Done())
            ++st.finished;
        }
      } else {
        pass_ok = cudaStreamSynchronize(static_cast<cudaStream_t>(
                      r.session->DeviceStream())) == cudaSuccess;
        if (!pass_ok)
          why = "prompt pass failed";
      }
    }
    if (!pass_ok) {
      r.failed = true;
      ++st.finished;
      note(why);
    }
    st.pass_ms = Ms(t0);
    break;
  }
  // 2. one decode round of up to 8 decoding requests
  std::vector<Request*> round;
  for (auto& r : requests_)
    if (r->Decoding() && round.size() < Session::kMaxBatch)
      round.push_back(r.get());
  if (!round.empty()) {
    const auto t0 = std::chrono::steady_clock::now();
    const size_t B = round.size();
    std::vector<Session*> sessions(B);
    std::vector<uint32_t> tokens(B), next(B), counts(B);
    std::vector<uint32_t> recent(B * kSampleMaxRecent);
    std::vector<uint64_t> seeds(B);
    for (size_t i = 0; i < B; ++i) {
      Request& r = *round[i];
      sessions[i] = r.session.get();
      tokens[i] = r.generated.back();
      r.Remember(tokens[i]);  // the token this round advances
      counts[i] = r.recent_count;
      std::copy(r.recent, r.recent + r.recent_count,
                recent.begin() + i * kSampleMaxRecent);
      seeds[i] = DrawSeed(r.seed, r.session->Position() + 1);
    }
    std::string why;
    if (Session::ForwardBatchSample(sessions, tokens, controls_, recent.data(),
                                    counts.data(), seeds.data(), next, &why)) {
      for (size_t i = 0; i < B; ++i) {
        round[i]->generated.push_back(next[i]);
        if (round[i]->Done())
          ++st.finished;
      }
      st.round_rows = uint32_t(B);
    } else {
      for (Request* r : round) {
        r->failed = true;
        ++st.finished;
      }
      note(why);
    }
    st.round_ms = Ms(t0);
  }
  return ok;
}

bool Scheduler::Idle() const {
  for (const auto& r : requests_)
    if (!r->Done())
      return false;
  return true;
}

std::span<const uint32_t> Scheduler::Tokens(int id) const {
  if (id < 0 || size_t(id) >= requests_.size())
    return {};
  return requests_[id]->generated;
}

bool Scheduler::Finished(int id) const {
  return id >= 0 && size_t(id) < requests_.size() && requests_[id]->Done();
}

bool Scheduler::Failed(int id) const {
  return id >= 0 && size_t(id) < requests_.size() && requests_[id]->failed;
}

}  // namespace lfm3
