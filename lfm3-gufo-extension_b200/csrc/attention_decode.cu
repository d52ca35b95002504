// Decode attention for every row of a round in one launch.
//
// Grid (kv_heads, splits, rows): a CTA owns one KV group of one row and a
// span of that row's keys, so ragged depths need no per-row launches. Every
// CTA normalises and rotates its group's query heads itself (cheap), and the
// CTA whose span ends at the row's position also stores the new K/V row in
// the ring. Keys stream through shared memory in tiles of 64 and an online
// softmax keeps FP32 scores, probabilities and accumulators (the decode
// precision of hip/ops.hip:1562-1691). With several spans, each CTA writes
// its maximum, denominator and unnormalised output, and whichever CTA of the
// group finishes last (a ticket, not a wait) merges them in span order and
// applies the gate (hip/ops.hip:1710-1728).
#include "attention.cuh"
#include "common.cuh"
#include "kernels.cuh"

namespace lfm3 {
namespace {

constexpr int kThreads = 128;
constexpr int kKPitch = 272;  // bytes per K row in shared memory
constexpr float kScoreScale = 0.0883883476483184405F;  // 1 / sqrt(128)

template <int G>
struct DecodeSmem {
  float q[G][kHeadDim];
  alignas(16) uint8_t k[kDecodeTile][kKPitch];
  alignas(16) __half v[kDecodeTile][kHeadDim];
  float s[kDecodeTile][G];  // scores, then probabilities
  float m[G], l[G], alpha[G];
  int last;
};

// RMSNorm (weight w) and RoPE of one 128-wide head held as pairs
// (i, i + 64) for i in {lane, lane + 32}; returns the rotated pairs.
__device__ __forceinline__ void norm_rope(float (&x0)[2], float (&x1)[2],
                                          const float* w, const float* freq,
                                          const float* factors, int position,
                                          float eps, int lane) {
  float squares = 0;
#pragma unroll
  for (int j = 0; j < 2; ++j)
    squares += x0[j] * x0[j] + x1[j] * x1[j];
  const float inv = 1.0F / sqrtf(warp_sum(squares) / 128.0F + eps);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = lane + 32 * j;
    const float a = (x0[j] * inv) * w[i], b = (x1[j] * inv) * w[i + 64];
    float angle = float(position) * freq[i];
    if (factors)
      angle /= factors[i];
    float sn, cs;
    sincosf(angle, &sn, &cs);
    x0[j] = a * cs - b * sn;
    x1[j] = b * cs + a * sn;
  }
}

template <int G>
__global__ void __launch_bounds__(kThreads)
    decode_attention_kernel(const __grid_constant__ DecodeAttentionParams p) {
  __shared__ DecodeSmem<G> s;
  const int g = blockIdx.x, split = blockIdx.y, r = blockIdx.z;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  grid_dependency_wait();
  allow_dependents();
  const bool op = p.rows == nullptr;
  const int position = op ? p.position : p.rows->position[r];
  const LayerState state =
      op ? LayerState{nullptr, const_cast<__half*>(p.ring_k),
                      const_cast<__half*>(p.ring_v), p.capacity, 0}
         : p.rows->layers[r][p.layer];
  const int capacity = state.capacity;
  const int first = p.window > 0 ? max(0, position + 1 - p.window) : 0;
  const int tiles = (position + 1 - first + kDecodeTile - 1) / kDecodeTile;
  const int max_splits = max(1, min(p.max_splits, kMaxDecodeSplits));
  const int per = (tiles + max_splits - 1) / max_splits;
  const int used = (tiles + per - 1) / per;  // decode_spans_used
  if (split >= used)
    return;
  const int begin = first + split * per * kDecodeTile;
  const int end = min(begin + per * kDecodeTile, position + 1);
  const size_t stride = size_t(p.kv_heads) * kHeadDim;

  // ---- query heads of this group (normalised, rotated, FP32)
  for (int h = warp; h < G; h += kThreads / 32) {
    const float* qr = p.q + size_t(r) * p.ldq + size_t(g * G + h) * kHeadDim;
    float x0[2] = {qr[lane], qr[lane + 32]};
    float x1[2] = {qr[lane + 64], qr[lane + 96]};
    if (!op)
      norm_rope(x0, x1, p.q_norm, p.freq, p.factors, position, p.eps, lane);
    s.q[h][lane] = x0[0];
    s.q[h][lane + 32] = x0[1];
    s.q[h][lane + 64] = x1[0];
    s.q[h][lane + 96] = x1[1];
  }
  // ---- the new K/V row goes to its ring slot (span holding `position`)
  if (!op && split == used - 1 && warp == 0) {
    const float* kr = p.k + size_t(r) * p.ldk + size_t(g) * kHeadDim;
    const float* vr = p.v + size_t(r) * p.ldk + size_t(g) * kHeadDim;
    float x0[2] = {kr[lane], kr[lane + 32]};
    float x1[2] = {kr[lane + 64], kr[lane + 96]};
    norm_rope(x0, x1, p.k_norm, p.freq, p.factors, position, p.eps, lane);
    const size_t slot = size_t(position % capacity) * stride +
                        size_t(g) * kHeadDim;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = lane + 32 * j;
      state.k[slot + i] = __float2half_rn(x0[j]);
      state.k[slot + i + 64] = __float2half_rn(x1[j]);
      state.v[slot + i] = __float2half_rn(vr[i]);
      state.v[slot + i + 64] = __float2half_rn(vr[i + 64]);
    }
  }
  if (tid < G) {
    s.m[tid] = -INFINITY;
    s.l[tid] = 0;
  }
  float acc[G];
#pragma unroll
  for (int h = 0; h < G; ++h)
    acc[h] = 0;
  __syncthreads();

  // ---- K and V rows of a tile (16-byte pieces, L1 bypassed: the current
  // row was just written by this CTA), loaded into registers one tile ahead
  constexpr int kPieces = kDecodeTile * 16 / kThreads;
  uint4 kr[kPieces], vr[kPieces];
  const auto load_tile = [&](int base) {
    const int n = min(kDecodeTile, end - base);
#pragma unroll
    for (int j = 0; j < kPieces; ++j) {
      const int c = tid + j * kThreads, key = c / 16, piece = c % 16;
      kr[j] = make_uint4(0, 0, 0, 0);
      vr[j] = kr[j];
      if (key < n) {
        const int t = base + key;
        const __half *ks = state.k, *vs = state.v;
        size_t row = size_t(t % capacity) * stride;
        if (op && t >= position) {
          ks = p.chunk_k;
          vs = p.chunk_v;
          row = size_t(t - position) * stride;
        }
        row += size_t(g) * kHeadDim;
        kr[j] = __ldcg(reinterpret_cast<const uint4*>(ks + row) + piece);
        vr[j] = __ldcg(reinterpret_cast<const uint4*>(vs + row) + piece);
      }
    }
  };
  if (begin < end)
    load_tile(begin);
  for (int base = begin; base < end; base += kDecodeTile) {
    const int n = min(kDecodeTile, end - base);
#pragma unroll
    for (int j = 0; j < kPieces; ++j) {
      const int c = tid + j * kThreads, key = c / 16, piece = c % 16;
      *reinterpret_cast<uint4*>(&s.k[key][piece * 16]) = kr[j];
      *reinterpret_cast<uint4*>(&s.v[key][piece * 8]) = vr[j];
    }
    __syncthreads();
    if (base + kDecodeTile < end)
      load_tile(base + kDecodeTile);  // in flight during this tile's math
    // ---- scores: thread owns key tid % 64 and half of the heads
    {
      const int t = tid % kDecodeTile, hs = tid / kDecodeTile;
      constexpr int kH = G / 2;
      float dot[kH];
#pragma unroll
      for (int j = 0; j < kH; ++j)
        dot[j] = 0;
      const uint4* krow = reinterpret_cast<const uint4*>(s.k[t]);
#pragma unroll 4
      for (int c = 0; c < 16; ++c) {
        const uint4 raw = krow[c];
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
        float kf[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __half22float2(h2[i]);
          kf[2 * i] = f.x;
          kf[2 * i + 1] = f.y;
        }
#pragma unroll
        for (int j = 0; j < kH; ++j) {
          const float* qh = s.q[hs * kH + j] + c * 8;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dot[j] = fmaf(qh[i], kf[i], dot[j]);
        }
      }
#pragma unroll
      for (int j = 0; j < kH; ++j)
        s.s[t][hs * kH + j] = t < n ? dot[j] * kScoreScale : -INFINITY;
    }
    __syncthreads();
    // ---- online softmax per head
    for (int h = warp; h < G; h += kThreads / 32) {
      const float a = s.s[lane][h], b = s.s[lane + 32][h];
      const float top = warp_max(fmaxf(a, b));
      const float old = s.m[h];
      const float next = fmaxf(old, top);
      const float pa = expf(a - next), pb = expf(b - next);
      s.s[lane][h] = pa;
      s.s[lane + 32][h] = pb;
      const float sum = warp_sum(pa + pb);
      if (lane == 0) {
        const float alpha = expf(old - next);  // 0 for the first tile
        s.alpha[h] = alpha;
        s.l[h] = s.l[h] * alpha + sum;
        s.m[h] = next;
      }
    }
    __syncthreads();
    // ---- P V: thread owns dimension tid of every head
    {
#pragma unroll
      for (int h = 0; h < G; ++h)
        acc[h] *= s.alpha[h];
      for (int t = 0; t < n; ++t) {
        const float vt = __half2float(s.v[t][tid]);
#pragma unroll
        for (int h = 0; h < G; ++h)
          acc[h] = fmaf(s.s[t][h], vt, acc[h]);
      }
    }
    __syncthreads();
  }

  const int d = tid;
  if (used == 1) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const int head = g * G + h;
      const float gate = p.gate[size_t(r) * p.ldg + head];
      const float y = (acc[h] / s.l[h]) / (1 + expf(-gate));
      if (p.out_split)
        store_split(p.out_split, r, p.heads * kHeadDim, head * kHeadDim + d, y);
      if (p.out_f32)
        p.out_f32[size_t(r) * p.heads * kHeadDim + head * kHeadDim + d] = y;
    }
    return;
  }
  // ---- several spans: publish this one, merge in the last CTA
  const auto part = [&](int sp, int head) {
    return p.partials +
           ((size_t(r) * p.heads + head) * kMaxDecodeSplits + sp) *
               (kHeadDim + 2);
  };
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float* out = part(split, g * G + h);
    if (d == 0) {
      out[0] = s.m[h];
      out[1] = s.l[h];
    }
    out[2 + d] = acc[h];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    unsigned* ticket = p.tickets + r * p.kv_heads + g;
    const unsigned old = atomicAdd(ticket, 1u);
    s.last = old == unsigned(used - 1);
    if (s.last)
      *ticket = 0;
  }
  __syncthreads();
  if (!s.last)
    return;
  __threadfence();
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const int head = g * G + h;
    float maximum = -INFINITY;
    for (int sp = 0; sp < used; ++sp)
      maximum = fmaxf(maximum, __ldcg(part(sp, head)));
    float sum = 0, value = 0;
    for (int sp = 0; sp < used; ++sp) {
      const float* pp = part(sp, head);
      const float w = expf(__ldcg(pp) - maximum);
      sum = fmaf(__ldcg(pp + 1), w, sum);
      value = fmaf(__ldcg(pp + 2 + d), w, value);
    }
    const float gate = p.gate[size_t(r) * p.ldg + head];
    const float y = (value / sum) / (1 + expf(-gate));
    if (p.out_split)
      store_split(p.out_split, r, p.heads * kHeadDim, head * kHeadDim + d, y);
    if (p.out_f32)
      p.out_f32[size_t(r) * p.heads * kHeadDim + head * kHeadDim + d] = y;
  }
}

template <int G>
cudaError_t launch_group(const DecodeAttentionParams& p, int rows,
                         cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t config = {};
  const int spans = p.span_grid > 0 && p.span_grid < kMaxDecodeSplits
                        ? p.span_grid
                        : kMaxDecodeSplits;
  config.gridDim = dim3(p.kv_heads, spans, rows);
  config.blockDim = dim3(kThreads);
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  config.attrs = attr;
  config.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelEx(&config, decode_attention_kernel<G>, p);
}

}  // namespace

int decode_spans_used(int position, int window, int max_splits) {
  const int first = window > 0 ? max(0, position + 1 - window) : 0;
  const int tiles = (position + 1 - first + kDecodeTile - 1) / kDecodeTile;
  const int splits = max(1, min(max_splits, kMaxDecodeSplits));
  const int per = (tiles + splits - 1) / splits;
  return (tiles + per - 1) / per;
}

size_t decode_attention_partial_floats(int heads) {
  return size_t(kMaxBatch) * heads * kMaxDecodeSplits * (kHeadDim + 2);
}

cudaError_t launch_decode_attention(const DecodeAttentionParams& p, int rows,
                                    cudaStream_t stream, bool pdl) {
  if (p.kv_heads <= 0 || p.heads % p.kv_heads || rows <= 0 ||
      rows > kMaxBatch)
    return cudaErrorInvalidValue;
  switch (p.heads / p.kv_heads) {
    case 2:
      return launch_group<2>(p, rows, stream, pdl);
    case 4:
      return launch_group<4>(p, rows, stream, pdl);
    case 8:
      return launch_group<8>(p, rows, stream, pdl);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace lfm3
