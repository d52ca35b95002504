// Token selection after a decode round: repetition penalty, top-k,
// temperature and a seeded draw. The device kernels (sampling.cu) and the
// host sampler (sample_host) share every function of this header, with
// every floating-point operation rounded the same way on both sides, so both
// pick the same token from the same logits.
//
// The reference selects tokens on the host with Gufo core's
// sampling::SamplerState (runner.cpp:268-296; defaults temperature 0.1,
// top-k 50, repeat penalty 1.1 at runner.cpp:31-35); that sampler is not part
// of the reference tree, so the rule here is this library's own, in the
// order llama.cpp's sampler chain applies the same three controls:
//   1. each distinct token of the row's recent tokens: l = l > 0 ? l / p : l * p
//   2. the top_k largest logits, ordered by (logit descending, id ascending)
//      through an order-preserving key of the float bits
//   3. w_i = exp((l_i - l_0) / T) in double precision (exp_sampling below),
//      S = w_0 + w_1 + ... in that order, u = uniform [0, 1) from the row's
//      seed, token = the first candidate whose running sum exceeds u * S
//      (the last candidate if rounding leaves none).
// Temperature 0 selects the largest penalised logit (lowest id on ties).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>

namespace lfm3 {

constexpr int kSampleMaxTopK = 64;     // candidates per row
constexpr int kSampleMaxRecent = 64;   // penalised tokens per row
constexpr int kSampleSegment = 4096;   // logits per first-stage CTA
constexpr int kSampleThreads = 256;    // 16 logits (or candidates) per thread
constexpr int kSamplePerThread = kSampleSegment / kSampleThreads;
// second stage: every segment's candidates in one CTA
constexpr int kSampleMaxCandidates = kSampleSegment;

// ---- rounding-exact arithmetic shared by host and device ---------------------
// Device code would contract a * b + c into one fused operation; the
// intrinsics keep each operation separately rounded, as on the host (x86-64
// SSE arithmetic, no contraction).
#if defined(__CUDA_ARCH__)
#define LFM3_DADD(a, b) __dadd_rn((a), (b))
#define LFM3_DSUB(a, b) __dsub_rn((a), (b))
#define LFM3_DMUL(a, b) __dmul_rn((a), (b))
#define LFM3_DDIV(a, b) __ddiv_rn((a), (b))
#define LFM3_FDIV(a, b) __fdiv_rn((a), (b))
#define LFM3_FMUL(a, b) __fmul_rn((a), (b))
#else
#define LFM3_DADD(a, b) ((a) + (b))
#define LFM3_DSUB(a, b) ((a) - (b))
#define LFM3_DMUL(a, b) ((a) * (b))
#define LFM3_DDIV(a, b) ((a) / (b))
#define LFM3_FDIV(a, b) ((a) / (b))
#define LFM3_FMUL(a, b) ((a) * (b))
#endif

__host__ __device__ inline uint32_t float_bits(float v) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(v);
#else
  uint32_t u;
  std::memcpy(&u, &v, 4);
  return u;
#endif
}
__host__ __device__ inline float bits_float(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float v;
  std::memcpy(&v, &u, 4);
  return v;
#endif
}

// Order-preserving key: a > b as floats (with -0 below +0) iff key(a) >
// key(b) as unsigned integers.
__host__ __device__ inline uint32_t sample_key(float v) {
  const uint32_t u = float_bits(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__host__ __device__ inline float key_value(uint32_t key) {
  return bits_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

// Repetition penalty of one logit (llama.cpp / CTRL rule).
__host__ __device__ inline float penalise(float v, float penalty) {
  return v > 0.0F ? LFM3_FDIV(v, penalty) : LFM3_FMUL(v, penalty);
}

// SplitMix64 (Steele, Lea and Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014): one output of the generator seeded with `seed`.
__host__ __device__ inline uint64_t splitmix64(uint64_t seed) {
  uint64_t z = seed + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
// Uniform double in [0, 1) with 53 random bits.
__host__ __device__ inline double sample_uniform(uint64_t seed) {
  return double(splitmix64(seed) >> 11) * 0x1.0p-53;
}

// exp(x) for x <= 0, written out so host and device round identically:
// Cody and Waite's argument reduction x = n ln2 + r (ln2 split into a 42-bit
// head, so n * head is exact, and a tail), the Taylor series of e^r to
// degree 13 by Horner's rule (|r| <= 0.35: truncation below 1e-17), and the
// scale 2^n assembled from its exponent bits. Relative error below 1e-15;
// 0 for x < -700 (where the weights vanish next to the largest one's 1).
__host__ __device__ inline double exp_sampling(double x) {
  if (!(x > -700.0))
    return 0.0;
  constexpr double kInvLn2 = 0x1.71547652b82fep+0;
  constexpr double kLn2Hi = 0x1.62e42fefa3800p-1;
  constexpr double kLn2Lo = 0x1.ef35793c76730p-45;
  // 1 / i! for i = 13 .. 0
  constexpr double kInvFactorial[14] = {
      0x1.6124613a86d09p-33, 0x1.1eed8eff8d898p-29, 0x1.ae64567f544e4p-26,
      0x1.27e4fb7789f5cp-22, 0x1.71de3a556c734p-19, 0x1.a01a01a01a01ap-16,
      0x1.a01a01a01a01ap-13, 0x1.6c16c16c16c17p-10, 0x1.1111111111111p-7,
      0x1.5555555555555p-5,  0x1.5555555555555p-3,  0x1.0000000000000p-1,
      0x1.0000000000000p+0,  0x1.0000000000000p+0};
#if defined(__CUDA_ARCH__)
  const double n = floor(LFM3_DADD(LFM3_DMUL(x, kInvLn2), 0.5));
#else
  const double n = __builtin_floor(LFM3_DADD(LFM3_DMUL(x, kInvLn2), 0.5));
#endif
  const double r =
      LFM3_DSUB(LFM3_DSUB(x, LFM3_DMUL(n, kLn2Hi)), LFM3_DMUL(n, kLn2Lo));
  double p = kInvFactorial[0];
#pragma unroll
  for (int i = 1; i < 14; ++i)
    p = LFM3_DADD(LFM3_DMUL(p, r), kInvFactorial[i]);
  // n in [-1010, 0]: 2^n is a normal double
  const uint64_t bits = uint64_t(int64_t(n) + 1023) << 52;
#if defined(__CUDA_ARCH__)
  const double scale = __longlong_as_double(static_cast<long long>(bits));
#else
  double scale;
  std::memcpy(&scale, &bits, 8);
#endif
  return LFM3_DMUL(p, scale);
}

// Weight of a candidate with logit v next to the largest candidate v0.
__host__ __device__ inline double sample_weight(float v, float v0,
                                                float temperature) {
  return exp_sampling(LFM3_DDIV(LFM3_DSUB(double(v), double(v0)),
                                double(temperature)));
}

// The draw over weights w[0..n) (largest first): index of the first
// candidate whose running sum exceeds u * S.
__host__ __device__ inline int sample_pick(const double* w, int n, double u) {
  double total = 0.0;
  for (int i = 0; i < n; ++i)
    total = LFM3_DADD(total, w[i]);
  const double target = LFM3_DMUL(u, total);
  double run = 0.0;
  for (int i = 0; i < n; ++i) {
    run = LFM3_DADD(run, w[i]);
    if (run > target)
      return i;
  }
  return n - 1;
}

// Selection controls (lfm3_sampler in include/lfm3_cuda.h).
struct SampleControls {
  float temperature;     // 0: greedy
  int top_k;             // 1..kSampleMaxTopK (1 when greedy)
  float repeat_penalty;  // 1: off
};

// Launch-time tables of up to kMaxBatch rows (passed by value).
struct SampleParams {
  const float* logits;  // [rows][ld]
  int rows, vocab, ld, segments;
  SampleControls c;
  uint32_t recent[8][kSampleMaxRecent];
  uint32_t recent_count[8];
  uint64_t seed[8];
  uint32_t* cand_key;  // [rows][segments][top_k]
  uint32_t* cand_id;
  uint32_t* out;       // [rows] selected tokens (device)
};

// Checks the controls of lfm3_sampler for a vocabulary and fills c (top_k
// is 1 at temperature 0). Returns null, or why they are refused.
const char* sample_controls(float temperature, uint32_t top_k, float penalty,
                            int vocab, SampleControls* c);

// Device bytes of the candidate scratch for `rows` rows.
inline size_t sample_scratch_bytes(int rows, int vocab, int top_k) {
  const int segments = (vocab + kSampleSegment - 1) / kSampleSegment;
  return size_t(rows) * segments * top_k * 2 * sizeof(uint32_t);
}

// Two kernels on `stream`: per-segment candidates, then the per-row pick.
cudaError_t launch_sample(const SampleParams& p, cudaStream_t stream);

// The same selection on the host for `rows` rows of host logits (the
// reference point of the device kernels' tests, and the path for callers
// that read logits to the host).
void sample_host(const float* logits, int rows, int vocab, size_t ld,
                 const SampleControls& c, const uint32_t* recent,
                 const uint32_t* recent_count, const uint64_t* seeds,
                 uint32_t* out);

}  // namespace lfm3
