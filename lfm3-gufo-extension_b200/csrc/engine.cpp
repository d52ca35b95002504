// Host engine: weight upload, sessions, prompt passes and decode rounds.
//
// The per-layer sequence follows Session::Impl::Run (engine.cpp:257-527 of
// the reference): sandwich norms around a convolution or gated-attention
// mixer and a SwiGLU FFN, live-row pruning after the last full-attention
// layer for prompt passes, and batched decode rounds that share every
// weight read between up to eight sessions.
#include "engine.hpp"

#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <atomic>
#include <map>
#include <mutex>
#include <stdexcept>
#include <thread>
#include <unordered_set>

#include "kernels.cuh"
#include "tensor_map.hpp"

// the residual norm reads a prompt projection's split partial sums in the
// projection's tile layout
static_assert(lfm3::kPrefillTileRows == 256 &&
                  lfm3::kPrefillTileTokens == 256 &&
                  lfm3::kSplitTileFloats ==
                      lfm3::kPrefillTileRows * lfm3::kPrefillTileTokens,
              "split partial layout");

namespace lfm3 {
namespace {

void Throw(cudaError_t status) {
  if (status != cudaSuccess)
    throw std::runtime_error(cudaGetErrorString(status));
}

// Geometry this build supports (config.cpp:39-45 plus the kernels' tiling).
std::string Validate(const lfm3_weights& w) {
  const auto& c = w.config;
  if (!c.n_layers || c.n_layers > LFM3_MAX_LAYERS || c.head_dim != 128 ||
      !c.heads || !c.hidden || !c.intermediate || !c.vocab || !c.context ||
      c.conv_width < 2 || c.conv_width > 32 || !c.window)
    return "unsupported LFM3 dimensions";
  if (c.hidden % 512 || c.intermediate % 512 || (c.heads * 128) % 512)
    return "LFM3 widths must be multiples of 512";
  if (c.hidden > 8192)
    return "LFM3 hidden width above 8192";
  for (uint32_t i = 0; i < c.n_layers; ++i) {
    const uint32_t h = c.kv_heads[i];
    if ((c.layer_type[i] == LFM3_CONV) != (h == 0))
      return "invalid LFM3 layer heads";
    if (h && (c.heads % h || (c.heads / h != 2 && c.heads / h != 4 &&
                              c.heads / h != 8)))
      return "LFM3 GQA group must be 2, 4 or 8";
  }
  // every matrix Q8_0, or every matrix BF16 (the numerical-reference
  // weights)
  const uint32_t type = w.output.type;
  if (type != LFM3_Q8_0 && type != LFM3_BF16)
    return "this build needs Q8_0 or BF16 matrices";
  const auto matrix = [type](const lfm3_tensor& t) {
    return t.data && t.type == type;
  };
  if (!matrix(w.embedding) || !matrix(w.output))
    return "the embedding and output matrices must share one type";
  for (uint32_t i = 0; i < c.n_layers; ++i) {
    const auto& l = w.layers[i];
    if (!matrix(l.gate) || !matrix(l.up) || !matrix(l.down))
      return "the FFN matrices must share the model's matrix type";
    if (c.layer_type[i] == LFM3_CONV) {
      if (!matrix(l.in_proj) || !matrix(l.out_proj) || !l.conv.data ||
          l.conv.type != LFM3_F32)
        return "invalid LFM3 convolution layer";
    } else if (!matrix(l.q) || !matrix(l.k) || !matrix(l.v) ||
               !matrix(l.attn_gate) || !matrix(l.attn_out) ||
               !l.q_norm.data || !l.k_norm.data) {
      return "invalid LFM3 attention layer";
    }
    if (!l.norm.data || !l.ffn_norm.data)
      return "missing LFM3 norm";
  }
  if (!w.output_norm.data || !w.rope_freqs.data)
    return "missing LFM3 output norm or RoPE factors";
  return {};
}

template <class F>
void VisitTensors(lfm3_weights& w, F f) {
  f(w.embedding);
  f(w.output);
  f(w.output_norm);
  f(w.rope_freqs);
  for (uint32_t i = 0; i < w.config.n_layers; ++i) {
    auto& l = w.layers[i];
    for (lfm3_tensor* t :
         {&l.norm, &l.ffn_norm, &l.post_norm, &l.post_ffn_norm, &l.gate, &l.up,
          &l.down, &l.conv, &l.in_proj, &l.out_proj, &l.q, &l.k, &l.v,
          &l.q_norm, &l.k_norm, &l.attn_gate, &l.attn_out})
      if (t->data)
        f(*t);
  }
}

int CeilDiv(int a, int b) { return (a + b - 1) / b; }

// Host payloads to device memory through pinned staging: reader threads
// copy pieces of the payloads (in host-address order, i.e. file order for a
// mapped checkpoint) into a pool of pinned buffers and queue each buffer's
// asynchronous copy to its device destination; a buffer is reused once its
// copy has completed (its event). Pageable memory copied by cudaMemcpy
// goes through one internal staging buffer per call from one thread; this
// keeps several host readers and the copy engine busy at once, the role of
// the reference's parallel reader (upload.cpp:33-68).
class StagedUpload {
public:
  static constexpr size_t kPiece = 32ull << 20;
  static constexpr int kBuffers = 6;

  struct Copy {
    const char* host;
    char* device;
    size_t bytes;
  };

  explicit StagedUpload(int readers) : readers_(std::max(1, readers)) {}

  void Add(const void* host, void* device, size_t bytes) {
    for (size_t off = 0; off < bytes; off += kPiece)
      copies_.push_back({static_cast<const char*>(host) + off,
                         static_cast<char*>(device) + off,
                         std::min(kPiece, bytes - off)});
  }

  // Runs every queued copy; throws on a CUDA failure (after the readers
  // have stopped and the queued copies have finished).
  void Run() {
    if (copies_.empty())
      return;
    cudaStream_t stream = nullptr;
    Throw(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    std::vector<void*> staging(kBuffers, nullptr);
    std::vector<cudaEvent_t> done(kBuffers, nullptr);
    cudaError_t failure = cudaSuccess;
    for (int b = 0; b < kBuffers && failure == cudaSuccess; ++b) {
      failure = cudaHostAlloc(&staging[b], kPiece, cudaHostAllocDefault);
      if (failure == cudaSuccess)
        failure = cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming);
    }
    if (failure == cudaSuccess) {
      std::vector<int> free_buffers;
      for (int b = 0; b < kBuffers; ++b)
        free_buffers.push_back(b);
      std::mutex mu;
      std::condition_variable cv;
      size_t next = 0;
      const auto reader = [&] {
        for (;;) {
          int b = -1;
          size_t i = 0;
          {
            std::unique_lock<std::mutex> lock(mu);
            cv.wait(lock, [&] {
              return !free_buffers.empty() || next == copies_.size() ||
                     failure != cudaSuccess;
            });
            if (next == copies_.size() || failure != cudaSuccess)
              return;
            b = free_buffers.back();
            free_buffers.pop_back();
            i = next++;
          }
          // the buffer's previous copy must have left it
          cudaError_t e = cudaEventSynchronize(done[b]);
          const Copy& c = copies_[i];
          if (e == cudaSuccess) {
            std::memcpy(staging[b], c.host, c.bytes);
            e = cudaMemcpyAsync(c.device, staging[b], c.bytes,
                                cudaMemcpyHostToDevice, stream);
          }
          if (e == cudaSuccess)
            e = cudaEventRecord(done[b], stream);
          {
            std::lock_guard<std::mutex> lock(mu);
            if (e != cudaSuccess && failure == cudaSuccess)
              failure = e;
            free_buffers.push_back(b);
          }
          cv.notify_all();
        }
      };
      std::vector<std::thread> threads;
      for (int t = 0; t < std::min<int>(readers_, kBuffers); ++t)
        threads.emplace_back(reader);
      for (auto& t : threads)
        t.join();
    }
    const cudaError_t sync = cudaStreamSynchronize(stream);
    if (failure == cudaSuccess)
      failure = sync;
    for (int b = 0; b < kBuffers; ++b) {
      if (done[b])
        cudaEventDestroy(done[b]);
      if (staging[b])
        cudaFreeHost(staging[b]);
    }
    cudaStreamDestroy(stream);
    Throw(failure);
  }

private:
  int readers_;
  std::vector<Copy> copies_;
};

}  // namespace

// ---- DeviceBuffer -------------------------------------------------------------
DeviceBuffer::DeviceBuffer(size_t bytes) : bytes_(bytes) {
  if (bytes)
    Throw(cudaMalloc(&data_, bytes));
}
DeviceBuffer::~DeviceBuffer() {
  if (data_)
    cudaFree(data_);
}
DeviceBuffer::DeviceBuffer(DeviceBuffer&& o) noexcept
    : data_(o.data_), bytes_(o.bytes_) {
  o.data_ = nullptr;
  o.bytes_ = 0;
}
DeviceBuffer& DeviceBuffer::operator=(DeviceBuffer&& o) noexcept {
  std::swap(data_, o.data_);
  std::swap(bytes_, o.bytes_);
  return *this;
}

// ---- Model ----------------------------------------------------------------------
Model::~Model() {
  if (error_host_)
    cudaFreeHost(error_host_);
}

std::shared_ptr<Model> Model::Load(const lfm3_weights& host,
                                   std::string* error) {
  try {
    const std::string problem = Validate(host);
    if (!problem.empty())
      throw std::invalid_argument(problem);
    std::shared_ptr<Model> m(new Model);
    m->device_ = host;
    int device = 0;
    Throw(cudaGetDevice(&device));
    Throw(cudaDeviceGetAttribute(&m->sms_, cudaDevAttrMultiProcessorCount,
                                 device));
    // Distinct payloads in host order (a mapped checkpoint's file order),
    // packed into <=128 MiB segments with 256-byte alignment
    // (upload.cpp:12-16, 33-68), filled through pinned staging.
    std::map<const void*, size_t> payloads;
    VisitTensors(m->device_, [&](lfm3_tensor& t) {
      auto& bytes = payloads[t.data];
      bytes = std::max(bytes, t.bytes);
    });
    constexpr size_t kSegment = 128ull << 20, kAlign = 256;
    std::map<const void*, void*> placed;
    StagedUpload upload(int(std::min(4u, std::max(1u, std::thread::hardware_concurrency()))));
    auto it = payloads.begin();
    while (it != payloads.end()) {
      size_t bytes = 0;
      auto end = it;
      while (end != payloads.end() &&
             (end == it || bytes + end->second <= kSegment)) {
        bytes += (end->second + kAlign - 1) / kAlign * kAlign;
        ++end;
      }
      m->segments_.emplace_back(bytes);
      char* dst = m->segments_.back().as<char>();
      for (; it != end; ++it) {
        upload.Add(it->first, dst, it->second);
        placed[it->first] = dst;
        dst += (it->second + kAlign - 1) / kAlign * kAlign;
      }
      m->weight_bytes_ += bytes;
    }
    upload.Run();
    VisitTensors(m->device_, [&](lfm3_tensor& t) { t.data = placed.at(t.data); });
    m->PackDecodeGroups();
    // RoPE frequencies: float(pow(double theta, -2i/D)), global then sliding
    // (hip/ops.hip:1045-1050, engine.cpp:225-232).
    float freq[128];
    const auto& c = host.config;
    for (int i = 0; i < 64; ++i) {
      freq[i] = float(std::pow(double(c.theta), double(-2.0F * i / 128)));
      freq[64 + i] =
          float(std::pow(double(c.theta_swa), double(-2.0F * i / 128)));
    }
    Throw(cudaHostAlloc(reinterpret_cast<void**>(&m->error_host_),
                        sizeof(unsigned), cudaHostAllocMapped));
    *m->error_host_ = 0;
    Throw(cudaHostGetDevicePointer(reinterpret_cast<void**>(&m->error_device_),
                                   m->error_host_, 0));
    m->freq_ = DeviceBuffer(sizeof(freq));
    Throw(cudaMemcpy(m->freq_.data(), freq, sizeof(freq),
                     cudaMemcpyHostToDevice));
    return m;
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return nullptr;
  }
}

// Packs every matrix group a decode round reads (Q8_0, or the BF16
// numerical-reference weights) into the decode projections' fragment order
// (q8_decode.cuh), from the device copies just uploaded, into one
// allocation (256-byte aligned groups).
void Model::PackDecodeGroups() {
  const auto& c = device_.config;
  const int H = int(c.hidden), F = int(c.intermediate), A = int(c.heads) * 128;
  struct Job {
    DecodeGroup* group;
    const uint8_t* src[4];
  };
  std::vector<Job> jobs;
  decode_.assign(c.n_layers, DecodeLayer{});
  const auto q8 = [](const lfm3_tensor& t) {
    return static_cast<const uint8_t*>(t.data);
  };
  const auto add = [&](DecodeGroup& g, int kind, int K,
                       std::initializer_list<const lfm3_tensor*> srcs) {
    g.layout = DecodeLayout{};
    g.layout.kind = kind;
    g.layout.K = K;
    g.layout.H = H;
    g.layout.n_src = int(srcs.size());
    g.layout.bf16 = bf16() ? 1 : 0;
    Job job{&g, {}};
    int j = 0;
    for (const lfm3_tensor* t : srcs) {
      g.layout.rows[j] = int(t->rows);
      job.src[j++] = q8(*t);
    }
    if (!decode_layout(g.layout, sms_))
      throw std::invalid_argument("decode projection shape not supported");
    jobs.push_back(job);
  };
  for (uint32_t i = 0; i < c.n_layers; ++i) {
    const auto& l = device_.layers[i];
    DecodeLayer& d = decode_[i];
    if (c.layer_type[i] == LFM3_CONV) {
      add(d.in_proj, kDecConv, H, {&l.in_proj});
      add(d.out_proj, kDecPlain, H, {&l.out_proj});
    } else {
      add(d.qkvg, kDecPlain, H, {&l.q, &l.k, &l.v, &l.attn_gate});
      add(d.attn_out, kDecPlain, A, {&l.attn_out});
    }
    add(d.gate_up, kDecSwiGLU, H, {&l.gate, &l.up});
    if (!bf16() && F % 1024 == 0 && F > kDecStagedK) {
      // down over its two column halves as two sources, two m-tiles per
      // tile: each input record serves two m-tiles; the residual norm adds
      // the halves' outputs in order
      DecodeGroup& g = d.down;
      g.layout = DecodeLayout{};
      g.layout.kind = kDecPlain;
      g.layout.K = F / 2;
      g.layout.H = H;
      g.layout.n_src = 2;
      const int row_bytes = F / 32 * 34;
      for (int j = 0; j < 2; ++j) {
        g.layout.rows[j] = int(l.down.rows);
        g.layout.src_ld[j] = row_bytes;
        g.layout.x_col[j] = j * (F / 2);
      }
      g.layout.x_ld = F;
      Job job{&g, {q8(l.down), q8(l.down) + (F / 2) / 32 * 34}};
      if (!decode_layout(g.layout, sms_) || g.layout.first_mtile[1] % g.layout.mt)
        throw std::invalid_argument("decode projection shape not supported");
      jobs.push_back(job);
    } else {
      add(d.down, kDecPlain, F, {&l.down});
    }
  }
  add(decode_head_, kDecPlain, H, {&device_.output});
  size_t total = 0;
  for (const Job& job : jobs)
    total += (decode_packed_bytes(job.group->layout) + 255) / 256 * 256;
  packed_ = DeviceBuffer(total);
  uint8_t* dst = packed_.as<uint8_t>();
  for (const Job& job : jobs) {
    job.group->data = dst;
    Throw(launch_decode_pack(job.group->layout, job.src, dst, nullptr));
    dst += (decode_packed_bytes(job.group->layout) + 255) / 256 * 256;
  }
  Throw(cudaDeviceSynchronize());
}

std::unique_ptr<Session> Model::CreateSession(uint32_t context,
                                              std::string* error) {
  try {
    if (!context || context > config().context)
      throw std::invalid_argument("invalid LFM3 context");
    return std::unique_ptr<Session>(
        new Session(shared_from_this(), context));
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return nullptr;
  }
}

// ---- Session ------------------------------------------------------------------
Session::Session(std::shared_ptr<Model> model, uint32_t context)
    : model_(std::move(model)), context_(context) {
  const auto& c = model_->config();
  const size_t H = c.hidden, F = c.intermediate, A = size_t(c.heads) * 128;
  const size_t R = kPrefillChunk;
  uint32_t kv_max = 0;
  for (uint32_t i = 0; i < c.n_layers; ++i)
    kv_max = std::max(kv_max, c.kv_heads[i]);
  const size_t KV = size_t(kv_max) * 128;
  Throw(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
  Throw(cudaEventCreateWithFlags(&round_done_, cudaEventDisableTiming));
  try {
    // recurrent state (engine.cpp:55-77)
    std::vector<LayerState> table(c.n_layers);
    for (uint32_t i = 0; i < c.n_layers; ++i) {
      State s;
      if (c.layer_type[i] == LFM3_CONV) {
        s.conv = DeviceBuffer(H * (c.conv_width - 1) * 4);
        Throw(cudaMemset(s.conv.data(), 0, s.conv.bytes()));
      } else {
        s.capacity = c.layer_type[i] == LFM3_SLIDING_ATTENTION
                         ? std::min(context, c.window)
                         : context;
        const size_t bytes = size_t(s.capacity) * c.kv_heads[i] * 128 * 2;
        s.k = DeviceBuffer(bytes);
        s.v = DeviceBuffer(bytes);
      }
      table[i] = {s.conv.as<float>(), s.k.as<__half>(), s.v.as<__half>(),
                  int(s.capacity), 0};
      states_.push_back(std::move(s));
    }
    layer_table_ = DeviceBuffer(table.size() * sizeof(LayerState));
    Throw(cudaMemcpy(layer_table_.data(), table.data(), layer_table_.bytes(),
                     cudaMemcpyHostToDevice));
    frontier_ = DeviceBuffer(H * 4);
    logits_ = DeviceBuffer(size_t(c.vocab) * 4);
    // workspace
    const size_t width = std::max({3 * H, F, A});
    ids_ = DeviceBuffer(R * 4);
    rows_ = DeviceBuffer(sizeof(DecodeRows));
    x_ = DeviceBuffer(R * H * 4);
    out_ = DeviceBuffer(R * H * 4);
    out2_ = DeviceBuffer(size_t(kMaxBatch) * H * 4);
    p_ = DeviceBuffer(R * 3 * H * 4);
    q_ = DeviceBuffer(R * A * 4);
    k_ = DeviceBuffer(R * KV * 4);
    v_ = DeviceBuffer(R * KV * 4);
    gate_ = DeviceBuffer(R * c.heads * 4);
    a_ = DeviceBuffer(R * std::max(A, H) * 4);
    ff_ = DeviceBuffer(R * F * 4);
    zf_ = DeviceBuffer(R * H * 4);
    split_partial_ = DeviceBuffer(kPrefillPartialFloats * 4);
    // FP16 row-scaled activations, or (BF16 models) three bf16 planes
    half_ = DeviceBuffer(R * width * 2 * (model_->bf16() ? 3 : 1));
    scale_ = DeviceBuffer(R * 4);
    z_split_ = DeviceBuffer(kMaxBatch * H * 4);
    a_split_ = DeviceBuffer(kMaxBatch * std::max(A, H) * 4);
    h_split_ = DeviceBuffer(kMaxBatch * F * 4);
    z32_ = DeviceBuffer(kMaxBatch * H * 4);
    batch_logits_ = DeviceBuffer(kMaxBatch * size_t(c.vocab) * 4);
    chunk_k_ = DeviceBuffer(R * KV * 2);
    chunk_v_ = DeviceBuffer(R * KV * 2);
    attn_partials_ =
        DeviceBuffer(decode_attention_partial_floats(c.heads) * 4);
    attn_tickets_ = DeviceBuffer(kMaxBatch * std::max(kv_max, 1u) * 4);
    Throw(cudaMemset(attn_tickets_.data(), 0, attn_tickets_.bytes()));
    prompt_scratch_ = DeviceBuffer(
        std::max<size_t>(prompt_attention_scratch_floats(c.heads, R, context),
                         1) *
        4);
    Throw(cudaMallocHost(reinterpret_cast<void**>(&host_rows_),
                         kRowTables * sizeof(DecodeRows)));
    {
      const int segments =
          int((c.vocab + kSampleSegment - 1) / kSampleSegment);
      const int top_k =
          std::max(1, std::min(kSampleMaxTopK, kSampleMaxCandidates / segments));
      sample_scratch_ =
          DeviceBuffer(sample_scratch_bytes(int(kMaxBatch), int(c.vocab), top_k));
      sample_out_ = DeviceBuffer(kMaxBatch * sizeof(uint32_t));
      Throw(cudaMallocHost(reinterpret_cast<void**>(&sample_host_),
                           kMaxBatch * sizeof(uint32_t)));
    }
    for (cudaEvent_t& e : rows_copied_)
      Throw(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    Throw(cudaEventCreateWithFlags(&ready_, cudaEventDisableTiming));
    Throw(cudaMallocHost(reinterpret_cast<void**>(&graph_rows_),
                         sizeof(DecodeRows)));
    Throw(cudaEventCreateWithFlags(&graph_rows_copied_,
                                   cudaEventDisableTiming));
    static std::atomic<uint64_t> next_uid{1};
    uid_ = next_uid++;
    Throw(cudaDeviceSynchronize());
  } catch (...) {
    if (host_rows_)
      cudaFreeHost(host_rows_);
    if (graph_rows_)
      cudaFreeHost(graph_rows_);
    if (sample_host_)
      cudaFreeHost(sample_host_);
    cudaStreamDestroy(stream_);
    throw;
  }
}

Session::~Session() {
  if (stream_) {
    cudaStreamSynchronize(stream_);
    cudaStreamDestroy(stream_);
  }
  for (cudaEvent_t e : events_)
    cudaEventDestroy(e);
  if (round_done_)
    cudaEventDestroy(round_done_);
  for (cudaEvent_t e : rows_copied_)
    if (e)
      cudaEventDestroy(e);
  if (ready_)
    cudaEventDestroy(ready_);
  if (host_rows_)
    cudaFreeHost(host_rows_);
  if (round_exec_)
    cudaGraphExecDestroy(round_exec_);
  if (graph_rows_)
    cudaFreeHost(graph_rows_);
  if (graph_rows_copied_)
    cudaEventDestroy(graph_rows_copied_);
  if (sample_host_)
    cudaFreeHost(sample_host_);
}

void Session::Check(cudaError_t status) {
  if (inject_after_ > 0 && --inject_after_ == 0)
    status = cudaErrorLaunchFailure;
  Throw(status);
}

template <class F>
void Session::Timed(int cls, F launch) {
  if (!profiling_) {
    launch();
    return;
  }
  while (events_.size() < events_used_ + 2) {
    cudaEvent_t e;
    Check(cudaEventCreate(&e));
    events_.push_back(e);
  }
  cudaEvent_t a = events_[events_used_++], b = events_[events_used_++];
  Check(cudaEventRecord(a, stream_));
  launch();
  Check(cudaEventRecord(b, stream_));
  pending_.push_back({cls, a, b});
}

void Session::CollectProfile() {
  for (const auto& p : pending_) {
    float ms = 0;
    Check(cudaEventElapsedTime(&ms, p.start, p.end));
    profile_ms_[p.cls] += ms;
    profile_launches_[p.cls] += 1;
  }
  pending_.clear();
  events_used_ = 0;
}

void Session::TakeProfile(double* ms, long long* launches) {
  for (int i = 0; i < kProfileClasses; ++i) {
    if (ms)
      ms[i] += profile_ms_[i];
    if (launches)
      launches[i] += profile_launches_[i];
    profile_ms_[i] = 0;
    profile_launches_[i] = 0;
  }
}

// ---- decode round -------------------------------------------------------------

// The first bytes of the next projection a launch asks into L2 (its CTAs
// become resident only after this launch's leave, and read these first).
constexpr size_t kDecodePrefetchBytes = size_t(8) << 20;

// Launches one projection of the round's rows over a packed decode group
// (Q8_0 or BF16 copies): the same outputs and epilogue as the GemvParams
// describe; `next`, when given, is the projection that follows it.
static cudaError_t RunDecode(const GemvParams& g, const DecodeGroup& group,
                             Model& model, cudaStream_t stream,
                             const DecodeGroup* next = nullptr) {
  DecodeParams p{};
  p.layout = group.layout;
  p.w = group.data;
  if (next && next->data) {
    p.prefetch = next->data;
    p.prefetch_bytes =
        std::min(kDecodePrefetchBytes, decode_packed_bytes(next->layout)) /
        16 * 16;
  }
  p.tokens = g.tokens;
  p.x = g.x;
  for (int j = 0; j < 4; ++j)
    p.o[j] = DecodeOut{g.o[j].out, g.o[j].ld};
  p.split_out = g.split_out;
  p.split_width = g.split_width;
  if (g.kind == kGemvSwiGLU) {
    p.f32_out = g.o[0].out;
    p.f32_ld = g.o[0].ld;
  }
  p.conv_w = g.conv_w;
  p.rows = g.rows;
  p.layer = g.layer;
  p.L = g.L;
  return launch_decode_gemv(p, decode_grid(p.layout, model.sms()), stream,
                            true);
}

static GemvOutput Out(const lfm3_tensor& w, float* out, int ld) {
  return {static_cast<const uint8_t*>(w.data), out, int(w.rows), ld};
}

void Session::LaunchLmHead(const void* split_rows, int rows, float* out) {
  const auto& w = model_->weights();
  const auto& c = w.config;
  GemvParams p{};
  p.kind = kGemvPlain;
  p.K = c.hidden;
  p.tokens = rows;
  p.n_out = 1;
  p.o[0] = Out(w.output, out, c.vocab);
  p.x = split_rows;
  Check(RunDecode(p, model_->decode_head(), *model_, stream_));
}

void Session::DecodeRound(std::span<Session* const> batch,
                          std::span<const uint32_t> tokens, bool logits,
                          const float* const* input_rows, bool rows_on_host) {
  const auto& w = model_->weights();
  const auto& c = w.config;
  const int B = int(batch.size());
  const int H = c.hidden, F = c.intermediate, A = c.heads * 128;
  cudaStream_t s = stream_;
  // a projection of the round's rows through the layer's packed decode
  // group (Q8_0 or BF16)
  // `next`: the projection that follows in the round (its first weights go
  // to L2 while this one finishes)
  const auto gemv = [&](GemvParams p, const DecodeGroup& group,
                        const DecodeGroup* next) {
    Timed(kDecodeProjection,
          [&] { Check(RunDecode(p, group, *model_, s, next)); });
  };
  // the first projection of the layer after layer i (the LM head after the
  // last layer when the round computes logits)
  const auto next_layer = [&](uint32_t i) -> const DecodeGroup* {
    if (i + 1 < c.n_layers) {
      const DecodeLayer& n = model_->decode_layer(i + 1);
      return c.layer_type[i + 1] == LFM3_CONV ? &n.in_proj : &n.qkvg;
    }
    return logits ? &model_->decode_head() : nullptr;
  };
  // an earlier round that returned without waiting and has finished reports
  // its device wait failures here
  if (model_->RoundErrors()) {
    model_->ClearRoundErrors();
    if (const unsigned e = take_device_error())
      throw std::runtime_error(
          "device wait gave up in an earlier round, code " + std::to_string(e));
  }
  DecodeRows rows{};
  rows.count = B;
  for (int r = 0; r < B; ++r) {
    rows.position[r] = int(batch[r]->position_);
    rows.token[r] = tokens[r];
    rows.layers[r] = batch[r]->layer_table_.as<LayerState>();
  }
  const DecodeRows* dev_rows = rows_.as<DecodeRows>();
  // each attention layer's key spans: about equal lengths over the round's
  // rows, about two CTAs (one wave) per SM; full-attention spans hold at
  // least 4 key tiles (fewer partial results to merge), sliding-window spans
  // may hold one (a window's 4 tiles spread over 4 SMs); {tiles per span,
  // spans used}
  std::vector<std::pair<int, int>> spans(c.n_layers, {0, 0});
  for (uint32_t i = 0; i < c.n_layers; ++i) {
    if (c.layer_type[i] == LFM3_CONV)
      continue;
    const int window =
        c.layer_type[i] == LFM3_SLIDING_ATTENTION ? int(c.window) : 0;
    long key_tiles = 0;
    for (int r = 0; r < B; ++r)
      key_tiles += decode_key_tiles(rows.position[r], window);
    const long slots = 2L * model_->sms();
    const int span_tiles = int(std::max(
        window ? 1L : 4L, (key_tiles * long(c.kv_heads[i]) + slots - 1) / slots));
    int span_grid = 0;
    for (int r = 0; r < B; ++r)
      span_grid = std::max(span_grid,
                           decode_spans_used(rows.position[r], window,
                                             DecodeAttentionParams{}.max_splits,
                                             span_tiles));
    spans[i] = {span_tiles, span_grid};
  }
  // the round's launches, after the copy of its row table from the pinned
  // `table`; `copied` is recorded once that copy is done
  const auto enqueue = [&](const DecodeRows* table, cudaEvent_t copied,
                           unsigned record_flags) {
    Check(cudaMemcpyAsync(rows_.data(), table, sizeof(DecodeRows),
                          cudaMemcpyHostToDevice, s));
    Check(cudaEventRecordWithFlags(copied, s, record_flags));
    float* x = x_.as<float>();
    float* out = out_.as<float>();
    void* z = z_split_.data();
    Timed(kRowKernels, [&] {
      Check(launch_embed_norm(w.embedding.data, w.embedding.type, nullptr,
                              reinterpret_cast<const uint32_t*>(
                                  reinterpret_cast<const char*>(dev_rows) +
                                  offsetof(DecodeRows, token)),
                              x,
                              static_cast<const float*>(w.layers[0].norm.data),
                              NormOut{nullptr, z, nullptr, nullptr}, B, H,
                              c.eps,
                              s, /*pdl=*/false));  // after all earlier work
    });
    // rows given as input embeddings replace their token rows in x, then the
    // first norm runs again over every row
    bool embedded = false;
    for (int r = 0; input_rows && r < B; ++r)
      if (input_rows[r]) {
        Check(cudaMemcpyAsync(x + size_t(r) * H, input_rows[r], size_t(H) * 4,
                              rows_on_host ? cudaMemcpyHostToDevice
                                           : cudaMemcpyDeviceToDevice,
                              s));
        embedded = true;
      }
    if (embedded)
      Timed(kRowKernels, [&] {
        Check(launch_residual_norm(
            nullptr, nullptr, x,
            static_cast<const float*>(w.layers[0].norm.data),
            NormOut{nullptr, z, nullptr, nullptr}, B, H, c.eps, s, false));
      });
    for (uint32_t i = 0; i < c.n_layers; ++i) {
      const auto& l = w.layers[i];
      const DecodeLayer& dl = model_->decode_layer(i);
      if (c.layer_type[i] == LFM3_CONV) {
        GemvParams p{};
        p.kind = kGemvConv;
        p.K = H;
        p.tokens = B;
        p.n_out = 1;
        p.o[0] = Out(l.in_proj, nullptr, 0);
        p.x = z;
        p.split_out = a_split_.data();
        p.split_width = H;
        p.conv_w = static_cast<const float*>(l.conv.data);
        p.rows = dev_rows;
        p.layer = int(i);
        p.H = H;
        p.L = int(c.conv_width);
        gemv(p, dl.in_proj, &dl.out_proj);
        GemvParams o{};
        o.kind = kGemvPlain;
        o.K = H;
        o.tokens = B;
        o.n_out = 1;
        o.o[0] = Out(l.out_proj, out, H);
        o.x = a_split_.data();
        gemv(o, dl.out_proj, &dl.gate_up);
      } else {
        const int kv = int(c.kv_heads[i]) * 128;
        GemvParams p{};
        p.kind = kGemvPlain;
        p.K = H;
        p.tokens = B;
        p.n_out = 4;
        p.o[0] = Out(l.q, q_.as<float>(), A);
        p.o[1] = Out(l.k, k_.as<float>(), kv);
        p.o[2] = Out(l.v, v_.as<float>(), kv);
        p.o[3] = Out(l.attn_gate, gate_.as<float>(), c.heads);
        p.x = z;
        gemv(p, dl.qkvg, &dl.attn_out);
        const bool swa = c.layer_type[i] == LFM3_SLIDING_ATTENTION;
        DecodeAttentionParams ap{};
        ap.q = q_.as<float>();
        ap.k = k_.as<float>();
        ap.v = v_.as<float>();
        ap.gate = gate_.as<float>();
        ap.ldq = A;
        ap.ldk = kv;
        ap.ldg = c.heads;
        ap.q_norm = static_cast<const float*>(l.q_norm.data);
        ap.k_norm = static_cast<const float*>(l.k_norm.data);
        ap.freq = model_->frequencies(swa);
        ap.factors =
            swa ? nullptr : static_cast<const float*>(w.rope_freqs.data);
        ap.rows = dev_rows;
        ap.layer = int(i);
        ap.heads = c.heads;
        ap.kv_heads = int(c.kv_heads[i]);
        ap.window = swa ? int(c.window) : 0;
        ap.span_tiles = spans[i].first;
        ap.span_grid = spans[i].second;
        // the round's first kernel starts only after every earlier kernel of
        // the front stream and of the batch sessions' streams
        ap.ring_settled = 1;
        ap.eps = c.eps;
        ap.out_split = a_split_.data();
        ap.partials = attn_partials_.as<float>();
        ap.tickets = attn_tickets_.as<unsigned>();
        Timed(kDecodeAttention,
              [&] { Check(launch_decode_attention(ap, B, s, true)); });
        GemvParams o{};
        o.kind = kGemvPlain;
        o.K = A;
        o.tokens = B;
        o.n_out = 1;
        o.o[0] = Out(l.attn_out, out, H);
        o.x = a_split_.data();
        gemv(o, dl.attn_out, &dl.gate_up);
      }
      Timed(kRowKernels, [&] {
        Check(launch_residual_norm(
            out, static_cast<const float*>(l.post_norm.data), x,
            static_cast<const float*>(l.ffn_norm.data),
            NormOut{nullptr, z, nullptr, nullptr}, B, H, c.eps, s, true));
      });
      GemvParams f{};
      f.kind = kGemvSwiGLU;
      f.K = H;
      f.tokens = B;
      f.n_out = 2;
      f.o[0] = Out(l.gate, nullptr, 0);
      f.o[1] = Out(l.up, nullptr, 0);
      f.x = z;
      f.split_out = h_split_.data();
      f.split_width = F;
      gemv(f, dl.gate_up, &dl.down);
      // down, over two column halves when its group is split (the second
      // half's rows go to out2_, added by the norm)
      const bool halves = dl.down.layout.x_ld != 0;
      GemvParams d{};
      d.kind = kGemvPlain;
      d.K = F;
      d.tokens = B;
      d.n_out = halves ? 2 : 1;
      d.o[0] = Out(l.down, out, H);
      if (halves)
        d.o[1] = Out(l.down, out2_.as<float>(), H);
      d.x = h_split_.data();
      gemv(d, dl.down, next_layer(i));
      const bool last = i + 1 == c.n_layers;
      const float* next = static_cast<const float*>(
          last ? w.output_norm.data : w.layers[i + 1].norm.data);
      Timed(kRowKernels, [&] {
        Check(launch_residual_norm(
            out, static_cast<const float*>(l.post_ffn_norm.data), x, next,
            NormOut{last ? z32_.as<float>() : nullptr, z, nullptr, nullptr}, B,
            H, c.eps, s, true, nullptr,
            halves ? out2_.as<float>() : nullptr));
      });
    }
    if (logits)
      Timed(kDecodeProjection,
            [&] { LaunchLmHead(z, B, batch_logits_.as<float>()); });
    // each session's frontier (and logits) rows, in one launch
    static_assert(kMaxRowCopies >= 2 * kMaxBatch, "round-end copies");
    RowCopies copies{};
    copies.error_out = model_->RoundErrorWord();
    for (int r = 0; r < B; ++r) {
      Session* row = batch[r];
      copies.src[copies.count] = z32_.as<float>() + size_t(r) * H;
      copies.dst[copies.count] = row->frontier_.as<float>();
      copies.floats[copies.count++] = H;
      if (logits) {
        copies.src[copies.count] =
            batch_logits_.as<float>() + size_t(r) * c.vocab;
        copies.dst[copies.count] = row->logits_.as<float>();
        copies.floats[copies.count++] = int(c.vocab);
      }
    }
    Check(launch_row_copies(copies, s, true));
  };
  bool embedded_rows = false;
  for (int r = 0; input_rows && r < B; ++r)
    embedded_rows = embedded_rows || input_rows[r];
  if (round_graphs_ && !profiling_ && inject_after_ == 0 && !embedded_rows) {
    std::vector<uint64_t> key{uint64_t(B), uint64_t(logits)};
    for (int r = 0; r < B; ++r)
      key.push_back(batch[r]->uid_);
    const size_t batch_words = key.size();
    for (const auto& sp : spans) {
      key.push_back(uint64_t(sp.first));
      key.push_back(uint64_t(sp.second));
    }
    const bool same_batch =
        round_exec_ && round_key_.size() == key.size() &&
        std::equal(key.begin(), key.begin() + batch_words, round_key_.begin());
    if (!(round_exec_ && key == round_key_) &&
        (same_batch || key == pending_key_) && !CaptureRound(enqueue, key))
      round_graphs_ = false;
    if (round_graphs_ && round_exec_ && key == round_key_) {
      Check(cudaEventSynchronize(graph_rows_copied_));
      *graph_rows_ = rows;
      note_launch(round_kernels_);
      Check(cudaGraphLaunch(round_exec_, s));
      return;
    }
    pending_key_ = key;
  }
  // direct launches: the row table goes through a rotating pinned slot whose
  // previous copy is done
  const int slot = rows_next_;
  rows_next_ = (rows_next_ + 1) % kRowTables;
  Check(cudaEventSynchronize(rows_copied_[slot]));
  host_rows_[slot] = rows;
  enqueue(&host_rows_[slot], rows_copied_[slot], cudaEventRecordDefault);
}

template <class Enqueue>
bool Session::CaptureRound(const Enqueue& enqueue,
                           const std::vector<uint64_t>& key) {
  cudaStream_t s = stream_;
  const unsigned long long before = launch_count();
  if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) !=
      cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  bool ok = true;
  try {
    enqueue(graph_rows_, graph_rows_copied_, cudaEventRecordExternal);
  } catch (const std::exception&) {
    ok = false;
  }
  cudaGraph_t graph = nullptr;
  const cudaError_t end = cudaStreamEndCapture(s, &graph);
  // launches recorded into the graph count when it replays
  note_launch(-int(launch_count() - before));
  const auto fail = [&] {
    if (graph)
      cudaGraphDestroy(graph);
    cudaGetLastError();
    return false;
  };
  if (!ok || end != cudaSuccess || !graph)
    return fail();
  size_t n = 0;
  if (cudaGraphGetNodes(graph, nullptr, &n) != cudaSuccess)
    return fail();
  std::vector<cudaGraphNode_t> nodes(n);
  if (n && cudaGraphGetNodes(graph, nodes.data(), &n) != cudaSuccess)
    return fail();
  int kernels = 0;
  for (cudaGraphNode_t node : nodes) {
    cudaGraphNodeType type;
    if (cudaGraphNodeGetType(node, &type) == cudaSuccess &&
        type == cudaGraphNodeTypeKernel)
      ++kernels;
  }
  // the same launches with another span plan update the executable graph in
  // place; anything else instantiates it afresh
  bool updated = false;
  if (round_exec_) {
    cudaGraphExecUpdateResultInfo info{};
    updated = cudaGraphExecUpdate(round_exec_, graph, &info) == cudaSuccess;
    if (!updated) {
      cudaGetLastError();
      cudaGraphExecDestroy(round_exec_);
      round_exec_ = nullptr;
    }
  }
  if (!updated && cudaGraphInstantiate(&round_exec_, graph, 0) != cudaSuccess) {
    round_exec_ = nullptr;
    return fail();
  }
  cudaGraphDestroy(graph);
  round_key_ = key;
  round_kernels_ = kernels;
  return true;
}

// ---- prompt pass --------------------------------------------------------------
void Session::Prompt(std::span<const uint32_t> tokens, bool want_logits,
                     std::span<const RowRun> runs, bool on_device) {
  const auto& w = model_->weights();
  const auto& c = w.config;
  const int n = int(tokens.size());
  const int H = c.hidden, F = c.intermediate, A = c.heads * 128;
  const int L = int(c.n_layers);
  cudaStream_t s = stream_;
  Check(cudaMemcpyAsync(ids_.data(), tokens.data(), tokens.size_bytes(),
                        cudaMemcpyHostToDevice, s));
  // every prompt kernel waits for its predecessor in-kernel, so each may
  // launch while the previous one finishes (programmatic dependent launch)
  constexpr bool kPdl = true;
  // live rows (engine.cpp:304-323): after the last full-attention layer
  // only the frontier row, plus conv_width - 1 rows per trailing conv.
  std::vector<int> live_in(L, n), live_out(L, n);
  {
    int need = 1;
    for (int i = L; i-- > 0;) {
      if (c.layer_type[i] == LFM3_SLIDING_ATTENTION)
        break;
      live_out[i] = std::min(n, need);
      if (c.layer_type[i] == LFM3_FULL_ATTENTION)
        break;
      need = std::min(n, need + int(c.conv_width) - 1);
      live_in[i] = need;
    }
  }
  float* x = x_.as<float>();
  float* out = out_.as<float>();
  __half* half = half_.as<__half>();
  float* scale = scale_.as<float>();
  const auto half_at = [&](int row, int width) { return half + size_t(row) * width; };
  // Q8_0 prompt projections read FP16 rows of the workspace (viewed as
  // [rows][K]) starting at row `first`; BF16 ones the FP32 rows in32 (p.tokens
  // rows of K), split into three exact bf16 planes of the workspace first
  const bool bf16 = model_->bf16();
  const size_t half_elems = half_.bytes() / 2;
  const auto prefill = [&](PrefillParams p, int first,
                           const float* in32 = nullptr) {
    p.partial = split_partial_.as<float>();
    int splits = 1;
    if (bf16) {
      const int plane_rows = int(kPrefillChunk);
      Timed(kPromptOther, [&] {
        Check(launch_split_bf16_rows(in32, half, p.tokens, p.K, plane_rows, s,
                                     kPdl));
      });
      p.bf16 = 1;
      p.scale = nullptr;
      p.row_max = nullptr;
      p.x_row0 = 0;
      Timed(kPromptProjection, [&] {
        Check(launch_q8_prefill(p, half, plane_rows, s, &splits, kPdl));
      });
      return splits;
    }
    p.x_row0 = first;
    Timed(kPromptProjection, [&] {
      Check(launch_q8_prefill(p, half, int(half_elems / size_t(p.K)), s,
                              &splits, kPdl));
    });
    return splits;
  };
  const auto other = [&](auto launch) { Timed(kPromptOther, launch); };
  const auto rows = [&](auto launch) { Timed(kRowKernels, launch); };
  float* zf = zf_.as<float>();
  const auto norm_out = [&](int row) {
    return bf16 ? NormOut{zf + size_t(row) * H, nullptr, nullptr, nullptr}
                : NormOut{nullptr, nullptr, half_at(row, H), scale + row};
  };
  const auto to_half = [&](const float* src, int row, int n_rows, int width) {
    if (!bf16)
      Timed(kPromptOther, [&] {
        Check(launch_half_rows(src, nullptr, half_at(row, width), scale + row,
                               n_rows, width, s, kPdl));
      });
  };
  // a projection into the residual branch: its output, or the partial sums
  // of its K splits, which the residual norm adds in split order
  struct Branch {
    const float* data;
    SplitBranch split;
    const SplitBranch* parts() const { return split.partial ? &split : nullptr; }
  };
  const auto plain = [&](int K, int rows, int first_row, const float* in32,
                         std::initializer_list<PrefillOutput> outs,
                         bool planes = false) {
    const Branch whole{outs.begin()->out, {}};
    PrefillParams p{};
    p.kind = kPrefillPlain;
    p.K = K;
    p.tokens = rows;
    p.n_out = int(outs.size());
    int j = 0;
    for (const auto& o : outs)
      p.o[j++] = o;
    p.scale = bf16 ? nullptr : scale + first_row;
    p.keep_splits = planes;
    const int splits = prefill(p, first_row, in32);
    return planes && splits > 1
               ? Branch{nullptr,
                        SplitBranch{split_partial_.as<float>(), p.scale, splits,
                                    (rows + kPrefillTileTokens - 1) /
                                        kPrefillTileTokens}}
               : whole;
  };
  const auto pout = [](const lfm3_tensor& t, float* o, int ld) {
    return PrefillOutput{static_cast<const uint8_t*>(t.data), o, int(t.rows),
                         ld};
  };
  // embedding + first norm over layer 0's input rows
  {
    const int o_in = n - live_in[0];
    rows([&] {
      Check(launch_embed_norm(w.embedding.data, w.embedding.type,
                              ids_.as<uint32_t>(), nullptr, x, nullptr,
                              NormOut{}, n, H, c.eps, s, kPdl));
    });
    // rows given as input embeddings replace their token rows
    for (const RowRun& run : runs)
      Check(cudaMemcpyAsync(x + run.first * H, run.data, run.count * H * 4,
                            on_device ? cudaMemcpyDeviceToDevice
                                      : cudaMemcpyHostToDevice,
                            s));
    rows([&] {
      Check(launch_residual_norm(
          nullptr, nullptr, x + size_t(o_in) * H,
          static_cast<const float*>(w.layers[0].norm.data),
          norm_out(o_in), live_in[0], H, c.eps, s, kPdl));
    });
  }
  for (int i = 0; i < L; ++i) {
    const auto& l = w.layers[i];
    const int rows_in = live_in[i], rows_out = live_out[i];
    const int o_in = n - rows_in, o = n - rows_out;
    Branch branch{};
    if (c.layer_type[i] == LFM3_CONV) {
      float* p = p_.as<float>();
      plain(H, rows_in, o_in, zf + size_t(o_in) * H,
            {pout(l.in_proj, p + size_t(o_in) * 3 * H, 3 * H)});
      float* a = a_.as<float>();
      other([&] {
        Check(launch_short_conv(p + size_t(o_in) * 3 * H,
                                static_cast<const float*>(l.conv.data),
                                states_[i].conv.as<float>(),
                                a + size_t(o_in) * H, rows_in, H,
                                int(c.conv_width), true, s, kPdl));
      });
      to_half(a + size_t(o) * H, o, rows_out, H);
      branch = plain(H, rows_out, o, a + size_t(o) * H,
                     {pout(l.out_proj, out + size_t(o) * H, H)}, true);
    } else {
      const int kvh = int(c.kv_heads[i]), kv = kvh * 128;
      const size_t stride = size_t(kv);
      const bool swa = c.layer_type[i] == LFM3_SLIDING_ATTENTION;
      float *q = q_.as<float>(), *k = k_.as<float>(), *v = v_.as<float>(),
            *g = gate_.as<float>();
      plain(H, n, 0, zf,
            {pout(l.q, q, A), pout(l.k, k, kv), pout(l.v, v, kv),
             pout(l.attn_gate, g, c.heads)});
      auto& st = states_[i];
      // full-attention rows never wrap: pack them in place in the cache
      __half* kc = swa ? chunk_k_.as<__half>()
                       : st.k.as<__half>() + size_t(position_) * stride;
      __half* vc = swa ? chunk_v_.as<__half>()
                       : st.v.as<__half>() + size_t(position_) * stride;
      other([&] {
        Check(launch_prompt_heads(
            q, k, v, A, kv, static_cast<const float*>(l.q_norm.data),
            static_cast<const float*>(l.k_norm.data), model_->frequencies(swa),
            swa ? nullptr : static_cast<const float*>(w.rope_freqs.data), kc,
            vc, n, c.heads, kvh, int(position_), c.eps, s, kPdl));
      });
      const int skip = n - std::min(n, rows_out);
      float* a = a_.as<float>();
      Timed(kPromptAttention, [&] {
        if (swa)
          Check(launch_prompt_attention(
              q + size_t(skip) * A, A, kc + size_t(skip) * stride,
              vc + size_t(skip) * stride, st.k.as<__half>(),
              st.v.as<__half>(), g + size_t(skip) * c.heads, c.heads,
              a + size_t(skip) * A, n - skip, c.heads, kvh,
              int(position_) + skip, int(st.capacity), int(c.window),
              prompt_scratch_.as<float>(), s, kPdl));
        else  // every key is in the cache already
          Check(launch_prompt_attention_tc(
              q + size_t(skip) * A, A, st.k.as<__half>(), st.v.as<__half>(),
              g + size_t(skip) * c.heads, c.heads, a + size_t(skip) * A,
              n - skip, c.heads, kvh, int(position_) + skip,
              int(st.capacity), prompt_scratch_.as<float>(), s, kPdl));
      });
      if (swa)
        other([&] {
          Check(launch_store_kv(kc, vc, st.k.as<__half>(), st.v.as<__half>(),
                                n, kv, int(position_), int(st.capacity), s,
                                kPdl));
        });
      to_half(a + size_t(o) * A, o, rows_out, A);
      branch = plain(A, rows_out, o, a + size_t(o) * A,
                     {pout(l.attn_out, out + size_t(o) * H, H)}, true);
    }
    rows([&] {
      Check(launch_residual_norm(
          branch.data, static_cast<const float*>(l.post_norm.data),
          x + size_t(o) * H, static_cast<const float*>(l.ffn_norm.data),
          norm_out(o), rows_out, H, c.eps, s, kPdl, branch.parts()));
    });
    if (bf16) {
      // h rows in FP32, split into bf16 planes by the down projection
      float* ff = ff_.as<float>();
      PrefillParams p{};
      p.kind = kPrefillSwiGLU;
      p.K = H;
      p.tokens = rows_out;
      p.n_out = 2;
      p.o[0] = pout(l.gate, ff + size_t(o) * F, F);
      p.o[1] = pout(l.up, nullptr, F);
      prefill(p, o, zf + size_t(o) * H);
      branch = plain(F, rows_out, o, ff + size_t(o) * F,
                     {pout(l.down, out + size_t(o) * H, H)}, true);
    } else {
      // h rows in FP32, then FP16 with per-row scales (half_rows finds each
      // row's maximum itself)
      float* ff = ff_.as<float>();
      PrefillParams p{};
      p.kind = kPrefillSwiGLU;
      p.K = H;
      p.tokens = rows_out;
      p.n_out = 2;
      p.o[0] = pout(l.gate, ff + size_t(o) * F, F);
      p.o[1] = pout(l.up, nullptr, F);
      p.scale = scale + o;
      prefill(p, o);
      other([&] {
        Check(launch_half_rows(ff + size_t(o) * F, nullptr, half_at(o, F),
                               scale + o, rows_out, F, s, kPdl));
      });
      branch = plain(F, rows_out, o, nullptr,
                     {pout(l.down, out + size_t(o) * H, H)}, true);
    }
    const bool last = i + 1 == L;
    rows([&] {
      Check(launch_residual_norm(
          branch.data, static_cast<const float*>(l.post_ffn_norm.data),
          x + size_t(o) * H,
          last ? nullptr
               : static_cast<const float*>(w.layers[i + 1].norm.data),
          last ? NormOut{} : norm_out(o), rows_out, H, c.eps, s, kPdl,
          branch.parts()));
    });
  }
  // frontier = output_norm(last row); logits from it when asked
  rows([&] {
    Check(launch_residual_norm(
        nullptr, nullptr, x + size_t(n - 1) * H,
        static_cast<const float*>(w.output_norm.data),
        NormOut{frontier_.as<float>(), z_split_.data(), nullptr, nullptr}, 1,
        H, c.eps, s, kPdl));
  });
  if (want_logits)
    Timed(kDecodeProjection,
          [&] { LaunchLmHead(z_split_.data(), 1, logits_.as<float>()); });
}

// After a round this session led has finished: its last kernel copied the
// device error word into the model's host-mapped word, so a round that went
// through needs no device read (a synchronous copy on every step).
void Session::ThrowRoundErrors() {
  if (!model_->RoundErrors())
    return;
  model_->ClearRoundErrors();
  const unsigned e = take_device_error();
  throw std::runtime_error("device wait gave up, code " + std::to_string(e));
}

// Waits for everything queued for this session (its own stream also waits
// for rounds other sessions led) and reports a device wait that gave up.
void Session::Settle() {
  Check(cudaStreamSynchronize(stream_));
  if (const unsigned e = take_device_error()) {
    poisoned_ = true;
    throw std::runtime_error("device wait gave up, code " + std::to_string(e));
  }
}

void Session::EnsureLogits() {
  if (logits_ready_)
    return;
  const auto& c = model_->config();
  Check(launch_split_rows(frontier_.as<float>(), z_split_.data(), 1,
                          int(c.hidden), stream_));
  LaunchLmHead(z_split_.data(), 1, logits_.as<float>());
  Check(cudaStreamSynchronize(stream_));
  logits_ready_ = true;
}

// ---- public API -----------------------------------------------------------------
bool Session::Forward(std::span<const uint32_t> tokens, std::span<float> logits,
                      std::string* error) {
  const auto& c = model_->config();
  try {
    if (poisoned_)
      throw std::runtime_error("session is poisoned; Reset it first");
    if (!logits.empty() && logits.size() != c.vocab)
      throw std::invalid_argument("logits must hold vocab floats");
    if (tokens.empty())
      throw std::invalid_argument("no tokens");
    if (size_t(position_) + tokens.size() > context_)
      throw std::invalid_argument("LFM3 context overflow");
    for (uint32_t t : tokens)
      if (t >= c.vocab)
        throw std::invalid_argument("invalid LFM3 token");
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return false;
  }
  return Advance(tokens, {}, false, logits, error);
}

bool Session::Advance(std::span<const uint32_t> ids,
                      std::span<const RowRun> runs, bool on_device,
                      std::span<float> logits, std::string* error) {
  try {
    if (hooks_)
      hooks_->BeforeWrite(position_, position_ + uint32_t(ids.size()));
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return false;
  }
  const auto& c = model_->config();
  try {
    for (size_t first = 0; first < ids.size(); first += kPrefillChunk) {
      const auto chunk =
          ids.subspan(first, std::min(kPrefillChunk, ids.size() - first));
      const bool last = first + chunk.size() == ids.size();
      // the embedding runs inside this chunk, relative to its first row
      std::vector<RowRun> in_chunk;
      for (const RowRun& run : runs) {
        const size_t a = std::max(run.first, first);
        const size_t b = std::min(run.first + run.count, first + chunk.size());
        if (a < b)
          in_chunk.push_back(
              {a - first, b - a, run.data + (a - run.first) * c.hidden});
      }
      if (chunk.size() == 1) {
        Session* self = this;
        const float* row = in_chunk.empty() ? nullptr : in_chunk[0].data;
        DecodeRound({&self, 1}, chunk, last && !logits.empty(), &row,
                    !on_device);
      } else {
        Prompt(chunk, last && !logits.empty(), in_chunk, on_device);
      }
      // the chunks queue back to back; the last one (every one when
      // profiling) is waited for and its device waits checked
      if (last || profiling_) {
        Check(cudaStreamSynchronize(stream_));
        if (const unsigned e = take_device_error())
          throw std::runtime_error("device wait gave up, code " +
                                   std::to_string(e));
        CollectProfile();
      }
      position_ += uint32_t(chunk.size());
    }
    logits_ready_ = !logits.empty();
    if (!logits.empty())
      Check(cudaMemcpy(logits.data(), logits_.data(), logits.size_bytes(),
                       cudaMemcpyDeviceToHost));
    return true;
  } catch (const std::exception& e) {
    poisoned_ = true;
    if (error)
      *error = e.what();
    return false;
  }
}

bool Session::ForwardEmbeddings(std::span<const float> rows, bool on_device,
                                std::span<float> logits, std::string* error) {
  const auto& c = model_->config();
  const size_t n = rows.size() / c.hidden;
  try {
    if (poisoned_)
      throw std::runtime_error("session is poisoned; Reset it first");
    if (!logits.empty() && logits.size() != c.vocab)
      throw std::invalid_argument("logits must hold vocab floats");
    if (!n || rows.size() % c.hidden || !rows.data())
      throw std::invalid_argument("embedding rows must be hidden floats each");
    if (size_t(position_) + n > context_)
      throw std::invalid_argument("LFM3 context overflow");
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return false;
  }
  const std::vector<uint32_t> ids(n, 0);
  const RowRun all{0, n, rows.data()};
  return Advance(ids, {&all, 1}, on_device, logits, error);
}

bool Session::ForwardInputs(std::span<const Input> inputs,
                            std::span<float> logits, std::string* error) {
  const auto& c = model_->config();
  std::vector<uint32_t> ids;
  std::vector<RowRun> runs;
  try {
    if (poisoned_)
      throw std::runtime_error("session is poisoned; Reset it first");
    if (!logits.empty() && logits.size() != c.vocab)
      throw std::invalid_argument("logits must hold vocab floats");
    for (const Input& in : inputs) {
      if (!in.tokens.empty() && !in.rows.empty())
        throw std::invalid_argument("an input run holds tokens or rows");
      for (uint32_t t : in.tokens)
        if (t >= c.vocab)
          throw std::invalid_argument("invalid LFM3 token");
      if (in.rows.size() % c.hidden)
        throw std::invalid_argument("embedding rows must be hidden floats each");
      if (!in.rows.empty())
        runs.push_back({ids.size(), in.rows.size() / c.hidden, in.rows.data()});
      ids.insert(ids.end(), in.tokens.begin(), in.tokens.end());
      ids.resize(ids.size() + in.rows.size() / c.hidden, 0);
    }
    if (ids.empty())
      throw std::invalid_argument("no inputs");
    if (size_t(position_) + ids.size() > context_)
      throw std::invalid_argument("LFM3 context overflow");
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return false;
  }
  return Advance(ids, runs, false, logits, error);
}

bool Session::ForwardBatch(std::span<Session* const> sessions,
                           std::span<const uint32_t> tokens,
                           std::span<const std::span<float>> logits,
                           std::string* error) {
  return Batch(sessions, tokens, logits, false, error);
}

bool Session::ForwardBatchInputs(std::span<Session* const> sessions,
                                 std::span<const uint32_t> tokens, bool logits,
                                 std::string* error) {
  return Batch(sessions, tokens, {}, logits, error);
}

bool Session::ForwardBatchInputs(std::span<Session* const> sessions,
                                 std::span<const uint32_t> tokens,
                                 std::span<const float* const> rows,
                                 bool logits, std::string* error) {
  return Batch(sessions, tokens, {}, logits, error, rows);
}

bool Session::Batch(std::span<Session* const> sessions,
                    std::span<const uint32_t> tokens,
                    std::span<const std::span<float>> logits,
                    bool device_logits, std::string* error,
                    std::span<const float* const> rows) {
  // an embedding row stands in for its session's token
  const auto embedded = [&](size_t r) { return r < rows.size() && rows[r]; };
  uint32_t ids[kMaxBatch] = {};
  // every check before any mutation (engine.cpp:1178-1199)
  try {
    if (sessions.empty() || sessions.size() > kMaxBatch)
      throw std::invalid_argument("batch must hold 1..8 sessions");
    if (tokens.size() != sessions.size() ||
        (!logits.empty() && logits.size() != sessions.size()))
      throw std::invalid_argument("one token (and logits span) per session");
    const auto& model = sessions.front()->model_;
    std::unordered_set<const Session*> seen;
    for (size_t r = 0; r < sessions.size(); ++r) {
      const Session* s = sessions[r];
      if (!s || s->model_ != model)
        throw std::invalid_argument("batch sessions must share one model");
      if (!seen.insert(s).second)
        throw std::invalid_argument("duplicate batch session");
      if (s->poisoned_)
        throw std::runtime_error("batch session is poisoned");
      if (s->position_ >= s->context_)
        throw std::invalid_argument("LFM3 context overflow");
      if (!embedded(r) && tokens[r] >= model->config().vocab)
        throw std::invalid_argument("invalid LFM3 token");
      ids[r] = embedded(r) ? 0 : tokens[r];
      if (!logits.empty() && !logits[r].empty() &&
          logits[r].size() != model->config().vocab)
        throw std::invalid_argument("logits must hold vocab floats");
    }
    if (!rows.empty() && rows.size() != sessions.size())
      throw std::invalid_argument("one input row (or null) per session");
    for (Session* s : sessions)
      if (s->hooks_)
        s->hooks_->BeforeWrite(s->position_, s->position_ + 1);
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return false;
  }
  Session* front = sessions.front();
  bool want = device_logits;
  for (const auto& l : logits)
    want = want || !l.empty();
  try {
    // all sessions' earlier work must be done before the front stream
    // touches their state: the front stream waits for it on the device
    for (Session* s : sessions)
      if (s != front) {
        front->Check(cudaEventRecord(s->ready_, s->stream_));
        front->Check(cudaStreamWaitEvent(front->stream_, s->ready_, 0));
      }
    front->DecodeRound(sessions, std::span<const uint32_t>(ids, sessions.size()),
                       want, rows.empty() ? nullptr : rows.data());
    // logits spans that are consecutive rows of one block take one copy of
    // the round's logits; otherwise one copy per session
    bool block = !logits.empty();
    for (size_t r = 0; r < logits.size() && block; ++r)
      block = logits[r].size() == logits[0].size() &&
              logits[r].data() == logits[0].data() + r * logits[0].size();
    if (block)
      front->Check(cudaMemcpyAsync(logits[0].data(),
                                   front->batch_logits_.data(),
                                   logits.size() * logits[0].size_bytes(),
                                   cudaMemcpyDeviceToHost, front->stream_));
    for (size_t r = 0; r < logits.size() && !block; ++r)
      if (!logits[r].empty())
        front->Check(cudaMemcpyAsync(logits[r].data(),
                                     sessions[r]->logits_.data(),
                                     logits[r].size_bytes(),
                                     cudaMemcpyDeviceToHost, front->stream_));
    // ForwardBatchInputs (no host logits, no profiling) returns once the
    // round is enqueued: every batch session's own stream waits for it on
    // the device; a device wait that gave up is reported by a host read,
    // prompt pass, reset or snapshot of these sessions (they synchronise
    // first), or by a round that starts after this one has finished (the
    // host-mapped error word its last kernel writes)
    if (logits.empty() && !front->profiling_) {
      front->Check(cudaEventRecord(front->round_done_, front->stream_));
      for (Session* s : sessions)
        if (s != front)
          front->Check(cudaStreamWaitEvent(s->stream_, front->round_done_, 0));
    } else {
      front->Check(cudaStreamSynchronize(front->stream_));
      front->ThrowRoundErrors();
      front->CollectProfile();
    }
    for (size_t r = 0; r < sessions.size(); ++r) {
      sessions[r]->position_ += 1;
      sessions[r]->logits_ready_ = want;
    }
    return true;
  } catch (const std::exception& e) {
    for (Session* s : sessions)
      s->poisoned_ = true;
    if (error)
      *error = e.what();
    return false;
  }
}

bool Session::ForwardBatchSample(std::span<Session* const> sessions,
                                 std::span<const uint32_t> tokens,
                                 const SampleControls& controls,
                                 const uint32_t* recent,
                                 const uint32_t* recent_count,
                                 const uint64_t* seeds,
                                 std::span<uint32_t> next,
                                 std::string* error) {
  // the selection's own checks, before the round mutates anything
  const char* refused = nullptr;
  if (sessions.empty() || sessions.size() > kMaxBatch || !sessions.front())
    refused = "batch must hold 1..8 sessions";
  else if (next.size() != sessions.size() || !recent || !recent_count ||
           !seeds)
    refused = "one selected token and one row of tables per session";
  const int vocab = refused ? 0 : int(sessions.front()->config().vocab);
  const int segments = (vocab + kSampleSegment - 1) / kSampleSegment;
  if (!refused && (controls.top_k < 1 || controls.top_k > kSampleMaxTopK ||
                   segments * controls.top_k > kSampleMaxCandidates))
    refused = "sampler top_k does not fit this vocabulary";
  for (size_t r = 0; r < sessions.size() && !refused; ++r) {
    if (recent_count[r] > uint32_t(kSampleMaxRecent))
      refused = "more than 64 recent tokens in a row";
    for (uint32_t j = 0; j < recent_count[r] && !refused; ++j)
      if (recent[r * kSampleMaxRecent + j] >= uint32_t(vocab))
        refused = "recent token outside the vocabulary";
  }
  if (refused) {
    if (error)
      *error = refused;
    return false;
  }
  if (!Batch(sessions, tokens, {}, true, error))
    return false;
  Session* front = sessions.front();
  const int B = int(sessions.size());
  try {
    SampleParams p{};
    p.rows = B;
    p.logits = front->batch_logits_.as<float>();
    p.vocab = vocab;
    p.ld = vocab;
    p.segments = segments;
    p.c = controls;
    for (int r = 0; r < B; ++r) {
      p.recent_count[r] = recent_count[r];
      p.seed[r] = seeds[r];
      std::copy(recent + size_t(r) * kSampleMaxRecent,
                recent + size_t(r) * kSampleMaxRecent + recent_count[r],
                p.recent[r]);
    }
    p.cand_key = front->sample_scratch_.as<uint32_t>();
    p.cand_id = p.cand_key + size_t(B) * segments * controls.top_k;
    p.out = front->sample_out_.as<uint32_t>();
    front->Timed(kRowKernels,
                 [&] { front->Check(launch_sample(p, front->stream_)); });
    front->Check(cudaMemcpyAsync(front->sample_host_, p.out,
                                 size_t(B) * sizeof(uint32_t),
                                 cudaMemcpyDeviceToHost, front->stream_));
    front->Check(cudaStreamSynchronize(front->stream_));
    front->ThrowRoundErrors();  // the selection kernels do not wait
    front->CollectProfile();
    std::copy(front->sample_host_, front->sample_host_ + B, next.begin());
    return true;
  } catch (const std::exception& e) {
    for (Session* s : sessions)
      s->poisoned_ = true;
    if (error)
      *error = e.what();
    return false;
  }
}

bool Session::SampleLogits(const SampleControls& controls,
                           const uint32_t* recent, uint32_t recent_count,
                           uint64_t seed, uint32_t* token,
                           std::string* error) {
  const int vocab = int(config().vocab);
  const int segments = (vocab + kSampleSegment - 1) / kSampleSegment;
  const char* refused = nullptr;
  if (poisoned_ || !position_)
    refused = "no LFM3 logit frontier to select from";
  else if (!token || (recent_count && !recent) ||
           recent_count > uint32_t(kSampleMaxRecent))
    refused = "invalid selection tables";
  else if (controls.top_k < 1 || controls.top_k > kSampleMaxTopK ||
           segments * controls.top_k > kSampleMaxCandidates)
    refused = "sampler top_k does not fit this vocabulary";
  for (uint32_t j = 0; j < recent_count && !refused; ++j)
    if (recent[j] >= uint32_t(vocab))
      refused = "recent token outside the vocabulary";
  if (refused) {
    if (error)
      *error = refused;
    return false;
  }
  try {
    EnsureLogits();
    SampleParams p{};
    p.rows = 1;
    p.logits = logits_.as<float>();
    p.vocab = vocab;
    p.ld = vocab;
    p.segments = segments;
    p.c = controls;
    p.recent_count[0] = recent_count;
    p.seed[0] = seed;
    std::copy(recent, recent + recent_count, p.recent[0]);
    p.cand_key = sample_scratch_.as<uint32_t>();
    p.cand_id = p.cand_key + size_t(segments) * controls.top_k;
    p.out = sample_out_.as<uint32_t>();
    Timed(kRowKernels, [&] { Check(launch_sample(p, stream_)); });
    Check(cudaMemcpyAsync(sample_host_, p.out, sizeof(uint32_t),
                          cudaMemcpyDeviceToHost, stream_));
    Check(cudaStreamSynchronize(stream_));
    if (const unsigned e = take_device_error())
      throw std::runtime_error("device wait gave up, code " +
                               std::to_string(e));
    *token = sample_host_[0];
    return true;
  } catch (const std::exception& e) {
    poisoned_ = true;
    if (error)
      *error = e.what();
    return false;
  }
}

bool Session::ReadHidden(std::span<float> hidden, std::string* error) {
  try {
    if (hidden.size() != model_->config().hidden)
      throw std::invalid_argument("hidden must hold hidden floats");
    Settle();
    Check(cudaMemcpy(hidden.data(), frontier_.data(), hidden.size_bytes(),
                     cudaMemcpyDeviceToHost));
    return true;
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return false;
  }
}

bool Session::ReadLogits(std::span<float> logits, std::string* error) {
  try {
    if (poisoned_)
      throw std::runtime_error("session is poisoned");
    if (logits.size() != model_->config().vocab)
      throw std::invalid_argument("logits must hold vocab floats");
    if (!position_)
      throw std::runtime_error("no row advanced yet");
    EnsureLogits();
    Settle();
    Check(cudaMemcpy(logits.data(), logits_.data(), logits.size_bytes(),
                     cudaMemcpyDeviceToHost));
    return true;
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return false;
  }
}

bool Session::Reset(std::string* error) {
  try {
    if (hooks_)
      hooks_->BeforeReset();
    Throw(cudaStreamSynchronize(stream_));
    const auto& c = model_->config();
    for (size_t i = 0; i < states_.size(); ++i)
      if (states_[i].conv.data())
        Throw(cudaMemsetAsync(states_[i].conv.data(), 0,
                              size_t(c.hidden) * (c.conv_width - 1) * 4,
                              stream_));
    // a launch that gave up part way (a poisoned pass) may have left the
    // decode attention's span tickets counted; clear them with the state
    Throw(cudaMemsetAsync(attn_tickets_.data(), 0, attn_tickets_.bytes(),
                          stream_));
    Throw(cudaStreamSynchronize(stream_));
    position_ = 0;
    logits_ready_ = false;
    poisoned_ = false;
    inject_after_ = 0;
    return true;
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return false;
  }
}

bool Session::PrepareLogits(std::string* error) {
  try {
    if (poisoned_)
      throw std::runtime_error("session is poisoned; Reset it first");
    if (!position_)
      throw std::invalid_argument("no row advanced yet");
    EnsureLogits();
    return true;
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return false;
  }
}

bool Session::BeginRestore(std::string* error) {
  // engine.cpp:1374-1379: queued work ends before the adapter writes the
  // state; the session stays incoherent until FinishRestore
  try {
    Throw(cudaStreamSynchronize(stream_));
    poisoned_ = true;
    return true;
  } catch (const std::exception& e) {
    poisoned_ = true;
    if (error)
      *error = e.what();
    return false;
  }
}

bool Session::FinishRestore(uint32_t position, std::string* error) {
  // engine.cpp:1380-1386: the adapter wrote frontier, logits and every
  // layer's state for `position` rows
  if (position > context_) {
    if (error)
      *error = "restored position exceeds the session context";
    return false;
  }
  position_ = position;
  logits_ready_ = true;
  poisoned_ = false;
  return true;
}

void* Session::ContinuationData(ContinuationTensor tensor, size_t layer) const {
  switch (tensor) {
    case ContinuationTensor::kLogits:
      return logits_.data();
    case ContinuationTensor::kFrontier:
      return frontier_.data();
    case ContinuationTensor::kConvolution:
      return layer < states_.size() ? states_[layer].conv.data() : nullptr;
    case ContinuationTensor::kKey:
      return layer < states_.size() ? states_[layer].k.data() : nullptr;
    case ContinuationTensor::kValue:
      return layer < states_.size() ? states_[layer].v.data() : nullptr;
  }
  return nullptr;
}

uint32_t Session::RingCapacity(size_t layer) const {
  return layer < states_.size() ? states_[layer].capacity : 0;
}

// ---- snapshot v2 (engine.cpp:1387-1574) ---------------------------------------
namespace {
constexpr uint32_t kSnapshotMagic = 0x334d464c, kSnapshotVersion = 2;
constexpr size_t kSnapshotHeaderBytes = 32;
void PutWord(uint8_t* data, size_t word, uint32_t value) {
  for (int i = 0; i < 4; ++i)
    data[word * 4 + i] = uint8_t(value >> (i * 8));
}
uint32_t GetWord(const uint8_t* data, size_t word) {
  uint32_t value = 0;
  for (int i = 0; i < 4; ++i)
    value |= uint32_t(data[word * 4 + i]) << (i * 8);
  return value;
}
}  // namespace

// FNV-1a over the configuration fields in ConfigSignature's order
// (engine.cpp:1403-1419): hidden, intermediate, vocab, heads, head_dim,
// window, conv_width, the bit patterns of eps, theta and theta_swa, then each
// layer's type and KV head count. The context is not part of it (header word
// 2 carries it), so a snapshot written by the reference's engine restores
// here and the other way round.
uint32_t SnapshotSignature(const lfm3_config& c) {
  uint32_t h = 2166136261u;
  const auto mix = [&](uint32_t v) {
    for (int i = 0; i < 4; ++i) {
      h ^= (v >> (8 * i)) & 0xffu;
      h *= 16777619u;
    }
  };
  const auto bits = [](float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
  };
  for (const uint32_t v :
       {c.hidden, c.intermediate, c.vocab, c.heads, c.head_dim, c.window,
        c.conv_width, bits(c.eps), bits(c.theta), bits(c.theta_swa)})
    mix(v);
  for (uint32_t i = 0; i < c.n_layers; ++i) {
    mix(c.layer_type[i]);
    mix(c.kv_heads[i]);
  }
  return h;
}

namespace {
size_t RowsKept(uint32_t position, uint32_t capacity) {
  return std::min(position, capacity);
}
}  // namespace

size_t Session::SnapshotBytes() const {
  const auto& c = model_->config();
  size_t bytes = kSnapshotHeaderBytes + size_t(c.hidden) * 4 + size_t(c.vocab) * 4;
  for (uint32_t i = 0; i < c.n_layers; ++i) {
    if (c.layer_type[i] == LFM3_CONV)
      bytes += size_t(c.hidden) * (c.conv_width - 1) * 4;
    else
      bytes += 2 * RowsKept(position_, states_[i].capacity) * c.kv_heads[i] *
               128 * 2;
  }
  return bytes;
}

std::vector<uint8_t> Session::SaveSnapshot() {
  // a poisoned session's state may be partly written (engine.cpp:1471-1472)
  if (poisoned_)
    throw std::runtime_error("cannot snapshot a poisoned LFM3 session");
  const auto& c = model_->config();
  std::vector<uint8_t> out(SnapshotBytes());
  if (position_)
    EnsureLogits();
  Throw(cudaStreamSynchronize(stream_));
  uint8_t* p = out.data();
  PutWord(p, 0, kSnapshotMagic);
  PutWord(p, 1, kSnapshotVersion);
  PutWord(p, 2, context_);
  PutWord(p, 3, position_);
  PutWord(p, 4, c.hidden);
  PutWord(p, 5, c.vocab);
  PutWord(p, 6, c.n_layers);
  PutWord(p, 7, SnapshotSignature(c));
  p += kSnapshotHeaderBytes;
  // an empty session has no frontier: zeros, as the reference writes
  if (position_) {
    Throw(cudaMemcpy(p, frontier_.data(), size_t(c.hidden) * 4,
                     cudaMemcpyDeviceToHost));
    Throw(cudaMemcpy(p + size_t(c.hidden) * 4, logits_.data(),
                     size_t(c.vocab) * 4, cudaMemcpyDeviceToHost));
  }
  p += (size_t(c.hidden) + c.vocab) * 4;
  for (uint32_t i = 0; i < c.n_layers; ++i) {
    const auto& s = states_[i];
    if (c.layer_type[i] == LFM3_CONV) {
      const size_t bytes = size_t(c.hidden) * (c.conv_width - 1) * 4;
      Throw(cudaMemcpy(p, s.conv.data(), bytes, cudaMemcpyDeviceToHost));
      p += bytes;
    } else {
      const size_t bytes =
          RowsKept(position_, s.capacity) * c.kv_heads[i] * 128 * 2;
      Throw(cudaMemcpy(p, s.k.data(), bytes, cudaMemcpyDeviceToHost));
      p += bytes;
      Throw(cudaMemcpy(p, s.v.data(), bytes, cudaMemcpyDeviceToHost));
      p += bytes;
    }
  }
  return out;
}

bool Session::RestoreSnapshot(std::span<const uint8_t> payload,
                              std::string* error) {
  const auto& c = model_->config();
  try {
    if (hooks_)
      hooks_->BeforeRestore();
    // nothing queued may still write this session's state
    Throw(cudaStreamSynchronize(stream_));
    if (payload.size() < kSnapshotHeaderBytes)
      throw std::invalid_argument("truncated LFM3 snapshot");
    const uint8_t* p = payload.data();
    const uint32_t position = GetWord(p, 3);
    if (GetWord(p, 0) != kSnapshotMagic || GetWord(p, 1) != kSnapshotVersion ||
        GetWord(p, 2) != context_ || position > context_ ||
        GetWord(p, 4) != c.hidden || GetWord(p, 5) != c.vocab ||
        GetWord(p, 6) != c.n_layers || GetWord(p, 7) != SnapshotSignature(c))
      throw std::invalid_argument("invalid LFM3 snapshot header");
    size_t bytes = kSnapshotHeaderBytes + size_t(c.hidden) * 4 +
                   size_t(c.vocab) * 4;
    for (uint32_t i = 0; i < c.n_layers; ++i)
      bytes += c.layer_type[i] == LFM3_CONV
                   ? size_t(c.hidden) * (c.conv_width - 1) * 4
                   : 2 * RowsKept(position, states_[i].capacity) *
                         c.kv_heads[i] * 128 * 2;
    if (payload.size() != bytes)
      throw std::invalid_argument("LFM3 snapshot size mismatch");
  } catch (const std::exception& e) {
    if (error)
      *error = e.what();
    return false;
  }
  try {
    Throw(cudaStreamSynchronize(stream_));
    const uint8_t* p = payload.data();
    const uint32_t position = GetWord(p, 3);
    p += kSnapshotHeaderBytes;
    Throw(cudaMemcpy(frontier_.data(), p, size_t(c.hidden) * 4,
                     cudaMemcpyHostToDevice));
    p += size_t(c.hidden) * 4;
    Throw(cudaMemcpy(logits_.data(), p, size_t(c.vocab) * 4,
                     cudaMemcpyHostToDevice));
    p += size_t(c.vocab) * 4;
    for (uint32_t i = 0; i < c.n_layers; ++i) {
      auto& s = states_[i];
      if (c.layer_type[i] == LFM3_CONV) {
        const size_t bytes = size_t(c.hidden) * (c.conv_width - 1) * 4;
        Throw(cudaMemcpy(s.conv.data(), p, bytes, cudaMemcpyHostToDevice));
        p += bytes;
      } else {
        const size_t bytes =
            RowsKept(position, s.capacity) * c.kv_heads[i] * 128 * 2;
        Throw(cudaMemcpy(s.k.data(), p, bytes, cudaMemcpyHostToDevice));
        p += bytes;
        Throw(cudaMemcpy(s.v.data(), p, bytes, cudaMemcpyHostToDevice));
        p += bytes;
      }
    }
    position_ = position;
    logits_ready_ = position > 0;
    poisoned_ = false;
    return true;
  } catch (const std::exception& e) {
    poisoned_ = true;
    if (error)
      *error = e.what();
    return false;
  }
}

}  // namespace lfm3
