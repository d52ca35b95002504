// Host engine for the LFM3 backbone step on one B200: the C++ counterpart of
// the reference's Model / Session (engine.hpp:17-163), driving the sm_100a
// kernels of this library on one CUDA stream per session.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cuda.h>

#include <cstdint>
#include <map>
#include <memory>
#include <mutex>
#include <span>
#include <string>
#include <vector>

#include "../../include/lfm3_types.h"
#include "decode_types.cuh"
#include "q8_decode.cuh"
#include "sampling.cuh"

namespace lfm3 {

class Session;

// Snapshot header word 7 (ConfigSignature, engine.cpp:1403-1419).
uint32_t SnapshotSignature(const lfm3_config& c);

// Installed by the continuation (component cache) adapter
// (continuation_hooks.hpp:5-16): every callback runs on the host before the
// session changes state or submits device work, and may throw to refuse it.
class ContinuationHooks {
public:
  virtual ~ContinuationHooks() = default;
  // Rows [first, end) are about to be written.
  virtual void BeforeWrite(uint32_t first, uint32_t end) = 0;
  virtual void BeforeReset() = 0;
  virtual void BeforeRestore() = 0;
};

// Owns one device allocation.
class DeviceBuffer {
public:
  DeviceBuffer() = default;
  explicit DeviceBuffer(size_t bytes);
  ~DeviceBuffer();
  DeviceBuffer(DeviceBuffer&& other) noexcept;
  DeviceBuffer& operator=(DeviceBuffer&& other) noexcept;
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  template <class T>
  T* as() const {
    return static_cast<T*>(data_);
  }
  void* data() const { return data_; }
  size_t bytes() const { return bytes_; }

private:
  void* data_ = nullptr;
  size_t bytes_ = 0;
};

// Which continuation component ContinuationData returns
// (engine.hpp:9-15, ContinuationTensor).
enum class ContinuationTensor { kLogits, kFrontier, kConvolution, kKey, kValue };

// A Q8_0 or BF16 matrix group in the decode projections' fragment order
// (q8_decode.cuh), packed once at load.
struct DecodeGroup {
  DecodeLayout layout{};
  const uint8_t* data = nullptr;
};
// The groups one decode round reads per layer: a conv layer's in_proj
// (with the convolution step) and out_proj, an attention layer's fused
// q / k / v / gate projection and attn_out, and every layer's gate + up
// (SwiGLU) and down.
struct DecodeLayer {
  DecodeGroup in_proj, out_proj, qkvg, attn_out, gate_up, down;
};

class Model : public std::enable_shared_from_this<Model> {
public:
  ~Model();
  // Copies the packed tensors of host weights into 256-byte aligned device
  // segments (upload.cpp:33-68); tied tensors share one copy. Returns null
  // with *error set on invalid geometry or a CUDA failure.
  static std::shared_ptr<Model> Load(const lfm3_weights& host,
                                     std::string* error = nullptr);
  std::unique_ptr<Session> CreateSession(uint32_t context,
                                         std::string* error = nullptr);
  const lfm3_config& config() const { return device_.config; }
  // The weights with device payload pointers.
  const lfm3_weights& weights() const { return device_; }
  const float* frequencies(bool sliding) const {
    return freq_.as<float>() + (sliding ? 64 : 0);
  }
  int sms() const { return sms_; }
  // The host-mapped round error word: nonzero once a decode round ended with
  // the device error word set (its device address goes to that round's last
  // kernel).
  unsigned RoundErrors() const {
    return *static_cast<volatile unsigned*>(error_host_);
  }
  void ClearRoundErrors() { *static_cast<volatile unsigned*>(error_host_) = 0; }
  unsigned* RoundErrorWord() const { return error_device_; }
  // BF16 numerical-reference matrices (else Q8_0)
  bool bf16() const { return device_.output.type == LFM3_BF16; }
  // Device bytes of the weight segments.
  size_t weight_bytes() const { return weight_bytes_; }
  // The packed decode groups of layer i and of the LM head.
  const DecodeLayer& decode_layer(uint32_t i) const { return decode_[i]; }
  const DecodeGroup& decode_head() const { return decode_head_; }
  // Device bytes of the packed decode copies.
  size_t packed_bytes() const { return packed_.bytes(); }

private:
  Model() = default;
  lfm3_weights device_{};
  std::vector<DeviceBuffer> segments_;
  DeviceBuffer freq_;  // [2][64]: global then sliding theta
  int sms_ = 148;
  // Host-mapped copy of the device error word, written by the last kernel
  // of every decode round, so a round can check its predecessors without a
  // device-to-host copy (host and device addresses of one pinned word)
  unsigned* error_host_ = nullptr;
  unsigned* error_device_ = nullptr;

  size_t weight_bytes_ = 0;
  // the decode groups, all in one allocation
  DeviceBuffer packed_;
  std::vector<DecodeLayer> decode_;
  DecodeGroup decode_head_;
  void PackDecodeGroups();
  friend class Session;
};

class Session {
public:
  static constexpr size_t kPrefillChunk = 512;  // engine.hpp:47
  static constexpr size_t kMaxBatch = 8;        // engine.hpp:48
  ~Session();

  // Advances tokens in passes of at most kPrefillChunk rows and, when
  // logits is not empty, writes the final row's logits (host memory).
  // Validates before any mutation; a device error poisons the session
  // (engine.cpp:882-938).
  bool Forward(std::span<const uint32_t> tokens, std::span<float> logits = {},
               std::string* error = nullptr);
  // One token per independent session (2..8, distinct, same model), sharing
  // every weight read; logits[i] (host) may be empty (engine.cpp:1160-1216).
  static bool ForwardBatch(std::span<Session* const> sessions,
                           std::span<const uint32_t> tokens,
                           std::span<const std::span<float>> logits,
                           std::string* error = nullptr);
  // ForwardBatchInputs (engine.hpp:107-114) for token rows: logits, when
  // requested, stay in each session's device buffer (ContinuationData
  // kLogits); DeviceHidden of every session is updated. Returns once the
  // round is queued (unless profiling): work a caller queues on a session's
  // DeviceStream runs after it, the session's host reads wait for it, and a
  // device wait that gave up is reported by the next call that waits.
  static bool ForwardBatchInputs(std::span<Session* const> sessions,
                                 std::span<const uint32_t> tokens, bool logits,
                                 std::string* error = nullptr);
  // The same with input embeddings: rows[i], when set, is session i's input
  // row (hidden floats in device memory, ready in this call's stream order),
  // otherwise tokens[i] is (engine.hpp:107-114).
  static bool ForwardBatchInputs(std::span<Session* const> sessions,
                                 std::span<const uint32_t> tokens,
                                 std::span<const float* const> rows,
                                 bool logits, std::string* error = nullptr);
  // Advances rows of input embeddings (hidden floats each) instead of token
  // ids: host memory, or device memory read in this session's stream order
  // when on_device (engine.hpp:115-120).
  bool ForwardEmbeddings(std::span<const float> rows, bool on_device = false,
                         std::span<float> logits = {},
                         std::string* error = nullptr);
  // A run of token ids or of host embedding rows (engine.hpp:121-125).
  struct Input {
    std::span<const uint32_t> tokens;
    std::span<const float> rows;
  };
  // Advances runs in order; adjacent runs share their passes, so a prompt
  // mixing text and embeddings reads the weights once per 512 rows
  // (engine.hpp:126-131).
  bool ForwardInputs(std::span<const Input> inputs,
                     std::span<float> logits = {},
                     std::string* error = nullptr);
  // The reference starts an NPU decode early; on the GPU there is nothing to
  // start before the token is advanced (engine.hpp:71-73).
  void Speculate(uint32_t) {}
  // Continuation components (engine.hpp:144-158): the hooks (not owned; null
  // removes them), the frontier's logits completed on this session's stream,
  // and a restore by direct writes to ContinuationData between BeginRestore
  // (waits for queued work, marks the session incoherent) and
  // FinishRestore(position).
  void SetContinuationHooks(ContinuationHooks* hooks) { hooks_ = hooks; }
  bool PrepareLogits(std::string* error = nullptr);
  bool BeginRestore(std::string* error = nullptr);
  bool FinishRestore(uint32_t position, std::string* error = nullptr);
  // A round followed by token selection on the device (sampling.cuh): the
  // runner's AdvanceBatch + SelectNext (runner.cpp:268-351) without the
  // logits' trip to the host. next[i] is the token selected from session
  // i's new logits with row i of the host tables (recent[i * 64 + j] for
  // j < recent_count[i], seeds[i]); the logits stay readable by ReadLogits.
  // Returns once the tokens are on the host.
  static bool ForwardBatchSample(std::span<Session* const> sessions,
                                 std::span<const uint32_t> tokens,
                                 const SampleControls& controls,
                                 const uint32_t* recent,
                                 const uint32_t* recent_count,
                                 const uint64_t* seeds,
                                 std::span<uint32_t> next,
                                 std::string* error = nullptr);
  // Token selection on the device from this session's own frontier logits
  // (a prompt pass's last row): the runner's SelectNext after Prefill
  // (runner.cpp:249-299) without the logits' trip to the host. recent holds
  // recent_count (<= 64) tokens. Returns once the token is on the host.
  bool SampleLogits(const SampleControls& controls, const uint32_t* recent,
                    uint32_t recent_count, uint64_t seed, uint32_t* token,
                    std::string* error = nullptr);
  // The final-normed hidden state / logits of the last advanced row.
  bool ReadHidden(std::span<float> hidden, std::string* error = nullptr);
  bool ReadLogits(std::span<float> logits, std::string* error = nullptr);
  const float* DeviceHidden() const { return frontier_.as<float>(); }
  void* DeviceStream() const { return stream_; }
  bool Reset(std::string* error = nullptr);
  uint32_t Position() const { return position_; }
  bool IsCoherent() const { return !poisoned_; }
  void* ContinuationData(ContinuationTensor tensor, size_t layer = 0) const;
  uint32_t RingCapacity(size_t layer) const;
  // Snapshot v2 (engine.cpp:1387-1574): 32-byte header, frontier, logits,
  // then per layer the convolution history or K and V rows in physical ring
  // order.
  size_t SnapshotBytes() const;
  std::vector<uint8_t> SaveSnapshot();
  bool RestoreSnapshot(std::span<const uint8_t> payload,
                       std::string* error = nullptr);
  uint32_t context() const { return context_; }
  const lfm3_config& config() const { return model_->config(); }
  // Fault injection for tests: the k-th subsequent CUDA call made by this
  // session's passes reports an error (0 disables).
  void InjectFailure(int after_calls) { inject_after_ = after_calls; }

  // Optional kernel timing by class, with events around every launch of this
  // session's passes (and rounds it leads). Events between launches
  // serialise them, so this is for a separate profiled pass, never for the
  // headline timing.
  enum ProfileClass {
    kDecodeProjection,  // q8_gemv
    kDecodeAttention,
    kRowKernels,        // embedding, norms, splits
    kPromptProjection,  // q8_prefill
    kPromptAttention,
    kPromptOther,       // heads, convolution, FP16 rows, ring store
    kProfileClasses
  };
  void SetProfiling(bool on) { profiling_ = on; }
  // Adds the accumulated milliseconds and launches per class and clears them.
  void TakeProfile(double* ms, long long* launches);

private:
  Session(std::shared_ptr<Model> model, uint32_t context);
  void Check(cudaError_t status);
  // Rows [first, first + count) of a pass taken from input embeddings.
  struct RowRun {
    size_t first, count;
    const float* data;
  };
  // Validated rows: ids (any valid id where a run supplies the row) and the
  // runs of embedding rows (host, or device when on_device).
  bool Advance(std::span<const uint32_t> ids, std::span<const RowRun> runs,
               bool on_device, std::span<float> logits, std::string* error);
  void Prompt(std::span<const uint32_t> tokens, bool logits,
              std::span<const RowRun> runs = {}, bool on_device = false);
  // rows[r], when set, replaces row r's token (hidden floats, device memory
  // unless rows_on_host)
  void DecodeRound(std::span<Session* const> batch,
                   std::span<const uint32_t> tokens, bool logits,
                   const float* const* rows = nullptr,
                   bool rows_on_host = false);
  void EnsureLogits();
  void Settle();
  static bool Batch(std::span<Session* const> sessions,
                    std::span<const uint32_t> tokens,
                    std::span<const std::span<float>> logits,
                    bool device_logits, std::string* error,
                    std::span<const float* const> rows = {});
  void LaunchLmHead(const void* split_rows, int rows, float* out);
  // a finished round's device wait failures (the host-mapped word), thrown
  void ThrowRoundErrors();

  std::shared_ptr<Model> model_;
  cudaStream_t stream_ = nullptr;
  uint32_t context_ = 0, position_ = 0;
  bool poisoned_ = false, logits_ready_ = false;
  ContinuationHooks* hooks_ = nullptr;
  int inject_after_ = 0;
  struct State {
    DeviceBuffer conv, k, v;
    uint32_t capacity = 0;
  };
  std::vector<State> states_;
  DeviceBuffer layer_table_;  // LayerState[n_layers]
  DeviceBuffer frontier_, logits_;
  // workspace (this session's passes, and rounds it leads)
  DeviceBuffer ids_, rows_, x_, out_,
      out2_ /* a K-split decode projection's second half */, p_, q_, k_, v_, gate_, a_, ff_,
      half_, scale_, z_split_, a_split_, h_split_, z32_, batch_logits_,
      chunk_k_, chunk_v_, attn_partials_,
      attn_tickets_, prompt_scratch_, split_partial_, zf_;

  // token selection of the rounds this session leads: candidates, the
  // selected tokens, and their pinned host copy
  DeviceBuffer sample_scratch_, sample_out_;
  uint32_t* sample_host_ = nullptr;
  // the rows of the rounds this session leads: kRowTables pinned tables in
  // turn, each reused once its copy to the device is done
  static constexpr int kRowTables = 4;
  DecodeRows* host_rows_ = nullptr;
  cudaEvent_t rows_copied_[kRowTables] = {};
  int rows_next_ = 0;
  // The decode round as a CUDA graph (rounds this session leads): captured
  // on the second round of a batch composition (sessions by id, width,
  // logits) and attention span plan, replayed while they hold, updated in
  // place when only the plan changes. Its row table is copied from
  // graph_rows_ (pinned), refilled once the previous replay's copy is done.
  uint64_t uid_ = 0;
  cudaGraphExec_t round_exec_ = nullptr;
  std::vector<uint64_t> round_key_, pending_key_;
  int round_kernels_ = 0;
  bool round_graphs_ = true;  // off after a capture that failed
  DecodeRows* graph_rows_ = nullptr;
  cudaEvent_t graph_rows_copied_ = nullptr;
  // this session's queued work, waited for by a round another session leads
  cudaEvent_t ready_ = nullptr;
  bool profiling_ = false;
  std::vector<cudaEvent_t> events_;
  // end of the last round this session led without waiting for it
  cudaEvent_t round_done_ = nullptr;
  size_t events_used_ = 0;
  struct Pending {
    int cls;
    cudaEvent_t start, end;
  };
  std::vector<Pending> pending_;
  double profile_ms_[kProfileClasses] = {};
  long long profile_launches_[kProfileClasses] = {};
  template <class F>
  void Timed(int cls, F launch);
  // Records a decode round's launches (enqueue) as this session's round
  // graph under `key`; false if capture or instantiation failed.
  template <class Enqueue>
  bool CaptureRound(const Enqueue& enqueue, const std::vector<uint64_t>& key);
  void CollectProfile();
  friend class Model;
};

}  // namespace lfm3
