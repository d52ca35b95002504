// Token selection on the device after a decode round (see sampling.cuh for
// the rule). Two kernels:
//
//   sample_candidates_kernel  grid (segments, rows): a CTA stages 4096 of a
//       row's logits in shared memory, applies the repetition penalty to the
//       row's distinct recent tokens in its range, and keeps its top_k
//       largest by a 4-pass radix select on the order-preserving keys (8 bits
//       a pass, shared-memory histograms), ties to the lower id; candidates
//       are written in id order.
//   sample_pick_kernel  grid (rows): the same select over every segment's
//       candidates, a rank sort of the top_k by (logit desc, id asc), the
//       weights in parallel and the draw by one thread.
//
// The logits of a round are L2-resident (the LM head wrote them just
// before), so the first stage reads them once at L2 bandwidth; no thread
// ever waits on another CTA.
#include <algorithm>
#include <cmath>
#include <numeric>
#include <vector>

#include "kernels.cuh"
#include "sampling.cuh"

namespace lfm3 {

namespace {

constexpr int kPer = kSamplePerThread;

struct SelectSmem {
  unsigned hist[256];
  unsigned warp_sums[kSampleThreads / 32];
  unsigned digit, remaining;
};

// Exclusive prefix sum over the block's threads in thread order; *total
// receives the sum over all threads.
__device__ unsigned block_exclusive_scan(unsigned v, SelectSmem& s,
                                         unsigned* total) {
  const int lane = threadIdx.x % 32, warp = threadIdx.x / 32;
  unsigned inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o)
      inc += t;
  }
  __syncthreads();  // earlier readers of warp_sums are done
  if (lane == 31)
    s.warp_sums[warp] = inc;
  __syncthreads();
  unsigned before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < kSampleThreads / 32; ++w) {
    const unsigned x = s.warp_sums[w];
    before += w < warp ? x : 0u;
    all += x;
  }
  *total = all;
  return before + inc - v;
}

// Flags the `want` largest keys among the block's valid entries (thread t
// owns positions t * kPer .. t * kPer + kPer - 1); equal keys go to the
// lower position. Radix select: each pass fixes 8 more bits of the
// want-th largest key from a histogram of the entries that match the bits
// fixed so far.
__device__ void select_top(const uint32_t (&key)[kPer],
                           const bool (&valid)[kPer], unsigned want,
                           SelectSmem& s, bool (&sel)[kPer]) {
  unsigned mine = 0, all = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    mine += valid[i] ? 1u : 0u;
  block_exclusive_scan(mine, s, &all);
  if (all <= want) {
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      sel[i] = valid[i];
    return;
  }
  uint32_t prefix = 0, mask = 0;
  unsigned remaining = want;  // entries still to take at or below the prefix
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += kSampleThreads)
      s.hist[b] = 0;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (valid[i] && (key[i] & mask) == prefix)
        atomicAdd(&s.hist[(key[i] >> shift) & 255u], 1u);
    __syncthreads();
    if (threadIdx.x < 32) {
      // lane l holds bins 8l .. 8l + 7; `above` counts the higher bins
      const int lane = threadIdx.x;
      unsigned own = 0;
#pragma unroll
      for (int b = 0; b < 8; ++b)
        own += s.hist[lane * 8 + b];
      unsigned from = own;  // this lane's bins and every higher one
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned t = __shfl_down_sync(0xFFFFFFFFu, from, o);
        if (lane + o < 32)
          from += t;
      }
      const unsigned above = from - own;
      if (above < remaining && remaining <= from) {
        unsigned cum = above;
        for (int b = 7; b >= 0; --b) {
          const unsigned h = s.hist[lane * 8 + b];
          if (cum + h >= remaining) {
            s.digit = unsigned(lane * 8 + b);
            s.remaining = remaining - cum;
            break;
          }
          cum += h;
        }
      }
    }
    __syncthreads();
    prefix |= s.digit << shift;
    mask |= 255u << shift;
    remaining = s.remaining;
  }
  // prefix is the want-th largest key: every larger key is taken, and the
  // first `remaining` copies of it in position order
  unsigned ties = 0, unused = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    ties += (valid[i] && key[i] == prefix) ? 1u : 0u;
  unsigned rank = block_exclusive_scan(ties, s, &unused);
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const bool tie = valid[i] && key[i] == prefix;
    sel[i] = valid[i] && (key[i] > prefix || (tie && rank < remaining));
    rank += tie ? 1u : 0u;
  }
}

__global__ void __launch_bounds__(kSampleThreads)
    sample_candidates_kernel(const __grid_constant__ SampleParams p) {
  __shared__ float vals[kSampleSegment];
  __shared__ SelectSmem s;
  const int seg = blockIdx.x, r = blockIdx.y, tid = threadIdx.x;
  const int base = seg * kSampleSegment;
  const int len = min(kSampleSegment, p.vocab - base);
  const float* row = p.logits + size_t(r) * p.ld + base;
  for (int i = tid; i < len; i += kSampleThreads)
    vals[i] = row[i];
  __syncthreads();
  // each distinct recent token once, by the thread of its first occurrence
  if (p.c.repeat_penalty != 1.0F && tid < int(p.recent_count[r])) {
    const uint32_t t = p.recent[r][tid];
    bool first = true;
    for (int j = 0; j < tid; ++j)
      first = first && p.recent[r][j] != t;
    if (first && t >= uint32_t(base) && t < uint32_t(base + len))
      vals[t - base] = penalise(vals[t - base], p.c.repeat_penalty);
  }
  __syncthreads();
  uint32_t key[kPer];
  bool valid[kPer], sel[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int pos = tid * kPer + i;
    valid[i] = pos < len;
    key[i] = valid[i] ? sample_key(vals[pos]) : 0u;
  }
  select_top(key, valid, unsigned(p.c.top_k), s, sel);
  unsigned count = 0, total = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    count += sel[i] ? 1u : 0u;
  unsigned slot = block_exclusive_scan(count, s, &total);
  const size_t out0 = (size_t(r) * p.segments + seg) * p.c.top_k;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (sel[i]) {
      p.cand_key[out0 + slot] = key[i];
      p.cand_id[out0 + slot] = uint32_t(base + tid * kPer + i);
      ++slot;
    }
}

__global__ void __launch_bounds__(kSampleThreads)
    sample_pick_kernel(const __grid_constant__ SampleParams p) {
  __shared__ SelectSmem s;
  __shared__ uint32_t top_key[kSampleMaxTopK], top_id[kSampleMaxTopK];
  __shared__ uint32_t sorted_key[kSampleMaxTopK], sorted_id[kSampleMaxTopK];
  __shared__ double w[kSampleMaxTopK];
  const int r = blockIdx.x, tid = threadIdx.x, K = p.c.top_k;
  const int positions = p.segments * K;  // <= kSampleMaxCandidates
  uint32_t key[kPer], id[kPer];
  bool valid[kPer], sel[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int pos = tid * kPer + i;
    const int seg = pos / K, j = pos % K;
    const int len = min(kSampleSegment, p.vocab - seg * kSampleSegment);
    valid[i] = pos < positions && j < len;
    key[i] = id[i] = 0;
    if (valid[i]) {
      const size_t at = (size_t(r) * p.segments + seg) * K + j;
      key[i] = p.cand_key[at];
      id[i] = p.cand_id[at];
    }
  }
  select_top(key, valid, unsigned(K), s, sel);
  unsigned count = 0, total = 0;
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    count += sel[i] ? 1u : 0u;
  unsigned slot = block_exclusive_scan(count, s, &total);
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (sel[i]) {
      top_key[slot] = key[i];
      top_id[slot] = id[i];
      ++slot;
    }
  __syncthreads();
  const int n = int(total);  // min(top_k, vocab)
  if (tid < n) {
    const uint32_t k = top_key[tid], d = top_id[tid];
    int rank = 0;
    for (int j = 0; j < n; ++j)
      rank += (top_key[j] > k || (top_key[j] == k && top_id[j] < d)) ? 1 : 0;
    sorted_key[rank] = k;
    sorted_id[rank] = d;
  }
  __syncthreads();
  if (p.c.temperature == 0.0F) {
    if (tid == 0)
      p.out[r] = sorted_id[0];
    return;
  }
  if (tid < n)
    w[tid] = sample_weight(key_value(sorted_key[tid]), key_value(sorted_key[0]),
                           p.c.temperature);
  __syncthreads();
  if (tid == 0)
    p.out[r] = sorted_id[sample_pick(w, n, sample_uniform(p.seed[r]))];
}

}  // namespace

const char* sample_controls(float temperature, uint32_t top_k, float penalty,
                            int vocab, SampleControls* c) {
  if (!std::isfinite(temperature) || temperature < 0.0F)
    return "sampler temperature must be finite and >= 0";
  if (!std::isfinite(penalty) || !(penalty > 0.0F))
    return "sampler repeat penalty must be finite and > 0";
  if (vocab < 1)
    return "sampler vocabulary is empty";
  const int k = temperature == 0.0F ? 1 : int(top_k);
  if (temperature != 0.0F && (top_k < 1 || top_k > uint32_t(kSampleMaxTopK)))
    return "sampler top_k must be 1..64";
  const int segments = (vocab + kSampleSegment - 1) / kSampleSegment;
  if (long(segments) * k > kSampleMaxCandidates)
    return "vocabulary too large for this top_k (segments x top_k > 4096)";
  c->temperature = temperature;
  c->top_k = k;
  c->repeat_penalty = penalty;
  return nullptr;
}

cudaError_t launch_sample(const SampleParams& p, cudaStream_t stream) {
  if (p.rows < 1 || p.rows > 8 || p.vocab < 1 || p.c.top_k < 1 ||
      p.c.top_k > kSampleMaxTopK ||
      p.segments != (p.vocab + kSampleSegment - 1) / kSampleSegment ||
      p.segments * p.c.top_k > kSampleMaxCandidates)
    return cudaErrorInvalidValue;
  for (int r = 0; r < p.rows; ++r)
    if (p.recent_count[r] > uint32_t(kSampleMaxRecent))
      return cudaErrorInvalidValue;
  cudaError_t e =
      launch_kernel(sample_candidates_kernel, dim3(p.segments, p.rows),
                    dim3(kSampleThreads), 0, stream, false, p);
  if (e != cudaSuccess)
    return e;
  return launch_kernel(sample_pick_kernel, dim3(p.rows), dim3(kSampleThreads),
                       0, stream, false, p);
}

void sample_host(const float* logits, int rows, int vocab, size_t ld,
                 const SampleControls& c, const uint32_t* recent,
                 const uint32_t* recent_count, const uint64_t* seeds,
                 uint32_t* out) {
  std::vector<float> v(vocab);
  std::vector<uint32_t> order(vocab);
  const int K = std::min(c.temperature == 0.0F ? 1 : c.top_k, vocab);
  for (int r = 0; r < rows; ++r) {
    std::copy(logits + size_t(r) * ld, logits + size_t(r) * ld + vocab,
              v.begin());
    const uint32_t* mine = recent + size_t(r) * kSampleMaxRecent;
    if (c.repeat_penalty != 1.0F)
      for (uint32_t j = 0; j < recent_count[r]; ++j) {
        const uint32_t t = mine[j];
        if (t < uint32_t(vocab) && std::find(mine, mine + j, t) == mine + j)
          v[t] = penalise(v[t], c.repeat_penalty);
      }
    std::iota(order.begin(), order.end(), 0u);
    std::partial_sort(order.begin(), order.begin() + K, order.end(),
                      [&](uint32_t a, uint32_t b) {
                        const uint32_t ka = sample_key(v[a]),
                                       kb = sample_key(v[b]);
                        return ka > kb || (ka == kb && a < b);
                      });
    if (c.temperature == 0.0F) {
      out[r] = order[0];
      continue;
    }
    double w[kSampleMaxTopK];
    for (int i = 0; i < K; ++i)
      w[i] = sample_weight(v[order[i]], v[order[0]], c.temperature);
    out[r] = order[sample_pick(w, K, sample_uniform(seeds[r]))];
  }
}

}  // namespace lfm3
