// Decode projections over the fragment-ordered Q8_0 copy; see q8_decode.cuh.
//
// A tile (kMT m-tiles of 16 rows over all K columns) belongs to one CTA from
// first load to epilogue; CTA i takes tiles i, i + G, i + 2G, ... The layout
// (decode_layout) picks kMT per shape so that the busiest CTA holds as few
// m-tiles as possible, which keeps every shape of the graded model within
// about 15 % of a perfect split with no cross-CTA fix-up.
//
// Per CTA a producer warp streams the tile's units (kUB Q8 blocks x kMT
// m-tiles, one contiguous run of the packed copy: 512 columns, or 1024 for
// one-m-tile tiles, so a unit is 17-35 KB) into a ring of shared-memory
// slots with one bulk copy each. The weights are constant, so it starts
// before the previous kernel in the stream has finished (programmatic
// dependent launch); the CTA holds most of an SM's shared memory, so the
// next projection's CTAs start as this one's exit (two co-resident CTAs of
// consecutive projections measured slower: they split the SM's bandwidth).
//
// Eight consumer warps take kUB / 8 blocks of each unit and, per block and
// m-tile:
//
//   A = the block's 16 x 32 codes: one 16-byte shared load per thread, four
//       byte permutes and four half2 subtractions (exact fp16 values q)
//   B = the input rows' hi and lo fp16 terms (x = hi + lo, 22 significant
//       bits) of up to 8 tokens, loaded from L2 a unit ahead, or from
//       shared memory when the CTA holds several tiles of a K <= 2048
//       projection (the producer copies the inputs in once, after the
//       ring's first weights and the dependency wait)
//   C = four m16n8k16 MMAs (two k16 halves, hi and lo chains) in FP32, then
//       acc += d * (hi + lo)
//
// i.e. the reference's per-block order "sum += d * (sum of q * x)"
// (hip/ops.hip:784-809) with FP32 accumulation. Warp sums merge through
// shared memory in warp order, so results never depend on timing.
#include <algorithm>

#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.cuh"
#include "q8_decode.cuh"

namespace lfm3 {

namespace {

template <bool kStaged>
struct DecodeSmem {
  static constexpr int kRing = kStaged ? kDecRingStaged : kDecRingBytes;
  alignas(128) uint8_t ring[kRing];
  // kStaged: the input records, token g's at g * kDecXRowBytes
  alignas(16) uint8_t x[kStaged ? kMaxBatch * kDecXRowBytes : 16];
  alignas(16) float red[kDecWarps][kDecMaxMtiles * 128];
  alignas(16) float tile[kDecMaxMtiles * 128];
  uint64_t full[kDecMaxSlots];
  uint64_t empty[kDecMaxSlots];
  uint64_t x_full[kDecMaxXChunks];  // kStaged: unit c's input columns landed
};

// Four biased codes (u = q + 128, one little-endian word) as two half2 of q,
// exactly: each byte goes under the fp16 exponent of 1024 (0x64uu = 1024 +
// u) and 1152 is subtracted.
__device__ __forceinline__ void biased_to_half2(uint32_t u, uint32_t& lo,
                                                uint32_t& hi) {
  lo = __byte_perm(u, 0x64646464u, 0x5150);
  hi = __byte_perm(u, 0x64646464u, 0x5352);
  const __half2 bias = __half2half2(__ushort_as_half(0x6480));  // 1152
  __half2 l = __hsub2(*reinterpret_cast<__half2*>(&lo), bias);
  __half2 h = __hsub2(*reinterpret_cast<__half2*>(&hi), bias);
  lo = *reinterpret_cast<uint32_t*>(&l);
  hi = *reinterpret_cast<uint32_t*>(&h);
}

// m16n8k16 with a zero accumulator input.
__device__ __forceinline__ void mma_f16_first(float (&d)[4],
                                              const uint32_t (&a)[4],
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1),
        "f"(0.0F));
}

// m16n8k16 bf16 x bf16 -> f32, accumulating into d.
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4],
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two input values given as fp16 hi and lo terms (x = hi + lo, exact in
// FP32) as three bf16 terms t1 + t2 + t3 == x exactly: each term is the
// round-to-nearest bf16 of what the earlier terms left (x carries at most
// 22 significant bits, bf16 eight).
__device__ __forceinline__ void split_bf16(uint32_t hi, uint32_t lo,
                                           uint32_t (&t)[3]) {
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&hi));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&lo));
  float r0 = a.x + b.x, r1 = a.y + b.y;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(r0, r1);
    t[i] = *reinterpret_cast<const uint32_t*>(&v);
    if (i < 2) {
      const float2 f = __bfloat1622float2(v);
      r0 -= f.x;
      r1 -= f.y;
    }
  }
}

// A convolution step's window (the weights and the row's history) read by
// the thread that will need it before the dependency wait: the row table
// and each session's history are complete before the round's first kernel,
// and only this launch's epilogue writes this layer's history.
constexpr int kConvPreMax = 8;  // widths up to this are preloaded
struct ConvPre {
  float w[kConvPreMax], h[kConvPreMax];
  bool ok;
};
template <int kKind, int kMT>
__device__ void conv_preload(const DecodeParams& p, int t, int tid,
                             ConvPre& pre) {
  pre.ok = false;
  if constexpr (kKind == kDecConv) {
    constexpr int kCh = 16 * (kMT / 3);
    const int tok = tid / kCh, c = tid % kCh, ch = t * kCh + c, L = p.L;
    if (tid >= kCh * 8 || tok >= p.tokens || ch >= p.layout.H ||
        L > kConvPreMax || t >= p.layout.tiles)
      return;
    const float* own = p.rows->layers[tok][p.layer].conv + size_t(ch) * (L - 1);
    const float* w = p.conv_w + size_t(ch) * L;
#pragma unroll
    for (int j = 0; j < kConvPreMax; ++j) {
      pre.w[j] = j < L ? w[j] : 0.0F;
      pre.h[j] = j < L - 1 ? own[j] : 0.0F;
    }
    pre.ok = true;
  }
}

template <int kKind, int kMT>
__device__ void decode_epilogue(const DecodeParams& p, const float* tile,
                                int t, int tid, const ConvPre& pre) {
  if constexpr (kKind == kDecPlain) {
    // token-major so consecutive threads store consecutive rows
    for (int e = tid; e < kMT * 128; e += kDecWarps * 32) {
      const int tok = e / (kMT * 16), rest = e % (kMT * 16);
      const int m = rest / 16, r = rest % 16;
      int j = 0, row0 = 0;
      if (tok >= p.tokens || !decode_mtile_source(p.layout, t, m, j, row0))
        continue;
      const int row = row0 + r;
      if (row < p.layout.rows[j])
        p.o[j].out[size_t(tok) * p.o[j].ld + row] = tile[m * 128 + r * 8 + tok];
    }
  } else if constexpr (kKind == kDecSwiGLU) {
    constexpr int kHalf = kMT / 2, kRows = 16 * kHalf;
    for (int e = tid; e < kRows * 8; e += kDecWarps * 32) {
      const int tok = e / kRows, r = e % kRows;
      const int row = t * kRows + r;
      if (tok >= p.tokens || row >= p.layout.rows[0])
        continue;
      const int gi = (r / 16) * 128 + (r % 16) * 8 + tok;
      const float g = tile[gi], u = tile[kHalf * 128 + gi];
      // BatchedSwiGLUActivationKernel's formula (hip/ops.hip:175-177)
      const float sig = 1.0F / (1.0F + expf(-g));
      const float h = (g * sig) * u;
      if (p.split_out)
        store_split(p.split_out, tok, p.split_width, row, h);
      if (p.f32_out)
        p.f32_out[size_t(tok) * p.f32_ld + row] = h;
    }
  } else {
    // ConvolutionStep (hip/ops.hip:1135-1151) per (channel, token): FMA
    // chain over the window oldest first, then gate by C; the history
    // shifts by one and keeps the newest B * x.
    constexpr int kThird = kMT / 3, kCh = 16 * kThird;
    const int L = p.L;
    for (int e = tid; e < kCh * 8; e += kDecWarps * 32) {
      const int tok = e / kCh, c = e % kCh;
      const int ch = t * kCh + c;
      if (tok >= p.tokens || ch >= p.layout.H)
        continue;
      const int bi = (c / 16) * 128 + (c % 16) * 8 + tok;
      const float b = tile[bi], cg = tile[kThird * 128 + bi],
                  x = tile[2 * kThird * 128 + bi];
      float* own = p.rows->layers[tok][p.layer].conv + size_t(ch) * (L - 1);
      const float* w = p.conv_w + size_t(ch) * L;
      const float current = b * x;
      float sum = 0;
      if (pre.ok && e == tid && t == int(blockIdx.x)) {
#pragma unroll
        for (int j = 0; j < kConvPreMax; ++j) {
          if (j < L - 1)
            sum = fmaf(pre.w[j], pre.h[j], sum);
          else if (j == L - 1)
            sum = fmaf(pre.w[j], current, sum);
        }
#pragma unroll
        for (int j = 0; j < kConvPreMax - 2; ++j)
          if (j < L - 2)
            own[j] = pre.h[j + 1];
      } else {
        for (int j = 0; j < L - 1; ++j)
          sum = fmaf(w[j], own[j], sum);
        sum = fmaf(w[L - 1], current, sum);
        for (int j = 0; j < L - 2; ++j)
          own[j] = own[j + 1];
      }
      own[L - 2] = current;
      store_split(p.split_out, tok, p.split_width, ch, sum * cg);
    }
  }
}

// Tile t's sums are in the consumer warps' acc: merge the warps in order,
// then the epilogue.
template <int kKind, int kMT, class Smem>
__device__ void decode_finish(const DecodeParams& p, Smem& s,
                              const float (&acc)[kMT][4], int t,
                              const ConvPre& pre) {
  constexpr int kThreads = kDecWarps * 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, cq = lane & 3;
  float2* mine = reinterpret_cast<float2*>(s.red[warp]);
#pragma unroll
  for (int m = 0; m < kMT; ++m) {
    mine[(m * 128 + g * 8 + 2 * cq) / 2] = make_float2(acc[m][0], acc[m][1]);
    mine[(m * 128 + (g + 8) * 8 + 2 * cq) / 2] =
        make_float2(acc[m][2], acc[m][3]);
  }
  named_barrier(1, kThreads);
  for (int e = tid; e < kMT * 128; e += kThreads) {
    float v = s.red[0][e];
#pragma unroll
    for (int q = 1; q < kDecWarps; ++q)
      v += s.red[q][e];
    s.tile[e] = v;
  }
  named_barrier(1, kThreads);
  decode_epilogue<kKind, kMT>(p, s.tile, t, tid, pre);
  named_barrier(1, kThreads);
}

template <int kKind, int kMT, int kUB, bool kStaged, bool kBf16>
__global__ void __launch_bounds__(kDecThreads, 1)
    decode_gemv_kernel(const __grid_constant__ DecodeParams p) {
  using Smem = DecodeSmem<kStaged>;
  constexpr int kRec = kBf16 ? kDecRecordBf16 : kDecRecord;
  constexpr int kPerWarp = kUB / kDecWarps;          // blocks per warp
  constexpr int kW = kMT * kUB * kRec;               // bytes per unit
  constexpr int kSlots = Smem::kRing / kW < kDecMaxSlots ? Smem::kRing / kW
                                                         : kDecMaxSlots;
  static_assert(kSlots >= 4 && kW % 16 == 0 && kPerWarp >= 1, "ring");
  static_assert(kDecThreads == (kDecWarps + 1) * 32, "consumers + producer");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], kDecWarps);
    }
    for (int i = 0; i < kDecMaxXChunks; ++i)
      mbar_init(&s.x_full[i], 1);
    fence_barrier_init();
  }
  __syncthreads();
  allow_dependents();
  const int C = p.layout.K / (32 * kUB);  // units per tile
  const int G = gridDim.x;

  if (warp == kDecWarps) {
    // ---- producer: the weights are constant, so the ring fills before the
    // dependency wait; staged inputs follow it
    if (lane != 0)
      return;
    int slot = 0, issued = 0;
    uint32_t phase = 0;
    bool x_sent = !kStaged;
    const uint64_t policy = l2_evict_first_policy();  // weights: read once
    // the inputs in unit-sized column chunks, each on its own barrier, so
    // the consumers start on unit 0 while the later chunks fly
    const auto send_x = [&] {
      grid_dependency_wait();
      const uint32_t row = uint32_t(p.layout.K) * 4;
      constexpr uint32_t chunk = 32 * kUB * 4;  // one unit's columns
      for (int c = 0; c < C; ++c) {
        mbar_arrive_expect_tx(&s.x_full[c], chunk * uint32_t(p.tokens));
        for (int g = 0; g < p.tokens; ++g)
          bulk_load(s.x + g * kDecXRowBytes + c * chunk,
                    static_cast<const uint8_t*>(p.x) + size_t(g) * row +
                        c * chunk,
                    chunk, &s.x_full[c]);
      }
      x_sent = true;
    };
    for (int t = blockIdx.x; t < p.layout.tiles; t += G)
      for (int c = 0; c < C; ++c) {
        if (!x_sent && issued == kSlots)
          send_x();
        ++issued;
        if (!mbar_wait(&s.empty[slot], phase ^ 1, kErrGemvEmptyWait))
          return;
        mbar_arrive_expect_tx(&s.full[slot], kW);
        bulk_load_hint(s.ring + slot * kW, p.w + (size_t(t) * C + c) * kW,
                       kW, &s.full[slot], policy);
        if (++slot == kSlots) {
          slot = 0;
          phase ^= 1;
        }
      }
    if (!x_sent)
      send_x();
    // this CTA's slice of the next projection's first weights into L2
    if (p.prefetch_bytes) {
      const size_t per = (p.prefetch_bytes / G + 15) & ~size_t(15);
      const size_t lo = per * blockIdx.x;
      const size_t hi =
          lo + per < p.prefetch_bytes ? lo + per : p.prefetch_bytes;
      for (size_t at = lo; at < hi; at += 65536)
        prefetch_l2(p.prefetch + at,
                    uint32_t(hi - at < 65536 ? hi - at : 65536));
    }
    return;
  }

  // ---- consumers
  ConvPre pre;
  conv_preload<kKind, kMT>(p, blockIdx.x, tid, pre);
  grid_dependency_wait();
  const int g = lane >> 2, cq = lane & 3;
  const bool live = g < p.tokens;
  const uint4* xr = static_cast<const uint4*>(p.x);
  // input records per row, and the first record of the tile's source
  const int records = (p.layout.x_ld ? p.layout.x_ld : p.layout.K) / 8;
  int xrec0 = 0;
  // the hi and lo input terms of token g for this warp's blocks of unit c
  struct Terms {
    uint4 hi[kPerWarp], lo[kPerWarp];
  };
  const auto fetch = [&](int c, Terms& x) {
#pragma unroll
    for (int i = 0; i < kPerWarp; ++i) {
      x.hi[i] = make_uint4(0, 0, 0, 0);
      x.lo[i] = x.hi[i];
      if (live) {
        const int kb = c * kUB + warp * kPerWarp + i;
        if constexpr (kStaged) {
          const uint4* rec = reinterpret_cast<const uint4*>(
              s.x + g * kDecXRowBytes + (kb * 4 + cq) * 32);
          x.hi[i] = rec[0];
          x.lo[i] = rec[1];
        } else {
          const uint4* rec =
              xr + (size_t(g) * records + xrec0 + kb * 4 + cq) * 2;
          x.hi[i] = __ldg(rec);
          x.lo[i] = __ldg(rec + 1);
        }
      }
    }
  };
  int slot = 0;
  uint32_t phase = 0;
  for (int t = blockIdx.x; t < p.layout.tiles; t += G) {
    float acc[kMT][4];
#pragma unroll
    for (int m = 0; m < kMT; ++m)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        acc[m][j] = 0;
    if constexpr (kKind == kDecPlain && !kStaged) {
      int j = 0, row0 = 0;
      decode_mtile_source(p.layout, t, 0, j, row0);
      xrec0 = p.layout.x_col[j] / 8;
    }
    Terms cur, next;
    if constexpr (!kStaged)
      fetch(0, cur);
    for (int c = 0; c < C; ++c) {
      if constexpr (kStaged) {
        // shared-memory terms of this unit, once its chunk has landed (the
        // first tile waits; the barriers stay complete for later tiles)
        if (t == int(blockIdx.x) &&
            !mbar_wait(&s.x_full[c], 0, kErrGemvFullWait))
          return;
        fetch(c, cur);
      } else if (c + 1 < C) {
        fetch(c + 1, next);
      }
      if (!mbar_wait(&s.full[slot], phase, kErrGemvFullWait))
        return;
      const uint8_t* base = s.ring + slot * kW;
#pragma unroll
      for (int i = 0; i < kPerWarp; ++i) {
        const uint4 h = cur.hi[i], l = cur.lo[i];
        const uint8_t* rec = base + (warp * kPerWarp + i) * (kMT * kRec);
        if constexpr (kBf16) {
          // the block's input as three exact bf16 terms, shared by its
          // m-tiles; three MMAs per k16 half accumulate straight into acc
          uint32_t b[4][3];
          split_bf16(h.x, l.x, b[0]);
          split_bf16(h.y, l.y, b[1]);
          split_bf16(h.z, l.z, b[2]);
          split_bf16(h.w, l.w, b[3]);
#pragma unroll
          for (int m = 0; m < kMT; ++m) {
            const uint8_t* q = rec + m * kRec;
            const uint4 u = *reinterpret_cast<const uint4*>(q + lane * 16);
            const uint4 v =
                *reinterpret_cast<const uint4*>(q + 512 + lane * 16);
            const uint32_t a1[4] = {u.x, v.x, u.y, v.y};  // columns 8c..8c+3
            const uint32_t a2[4] = {u.z, v.z, u.w, v.w};  // 8c+4..8c+7
#pragma unroll
            for (int j = 0; j < 3; ++j) {
              mma_bf16(acc[m], a1, b[0][j], b[1][j]);
              mma_bf16(acc[m], a2, b[2][j], b[3][j]);
            }
          }
          continue;
        }
#pragma unroll
        for (int m = 0; m < kMT; ++m) {
          const uint8_t* r = rec + m * kDecRecord;
          const uint4 w = *reinterpret_cast<const uint4*>(r + lane * 16);
          const uint32_t sc =
              *reinterpret_cast<const uint32_t*>(r + 512 + g * 4);
          uint32_t a1[4], a2[4];
          biased_to_half2(w.x, a1[0], a1[2]);  // row g, columns 8cq .. 8cq+3
          biased_to_half2(w.z, a1[1], a1[3]);  // row g + 8
          biased_to_half2(w.y, a2[0], a2[2]);  // row g, columns 8cq+4 .. +7
          biased_to_half2(w.w, a2[1], a2[3]);  // row g + 8
          float ch[4], cl[4];
          mma_f16_first(ch, a1, h.x, h.y);
          mma_f16_first(cl, a1, l.x, l.y);
          mma_f16(ch, a2, h.z, h.w);
          mma_f16(cl, a2, l.z, l.w);
          const float2 d =
              __half22float2(*reinterpret_cast<const __half2*>(&sc));
          acc[m][0] = fmaf(d.x, ch[0] + cl[0], acc[m][0]);
          acc[m][1] = fmaf(d.x, ch[1] + cl[1], acc[m][1]);
          acc[m][2] = fmaf(d.y, ch[2] + cl[2], acc[m][2]);
          acc[m][3] = fmaf(d.y, ch[3] + cl[3], acc[m][3]);
        }
      }
      __syncwarp();
      if (lane == 0)
        mbar_arrive(&s.empty[slot]);
      if (++slot == kSlots) {
        slot = 0;
        phase ^= 1;
      }
      if constexpr (!kStaged)
        cur = next;
    }
    decode_finish<kKind, kMT>(p, s, acc, t, pre);
  }
}

// ---- packing -------------------------------------------------------------------
// BF16: lane l = 4g + c of a record writes row g's columns 8c..8c+7 of the
// block at 16 l and row g + 8's at 512 + 16 l (zeros for padding rows).
__global__ void decode_pack_bf16_kernel(const DecodeLayout l, const uint8_t* s0,
                                        const uint8_t* s1, const uint8_t* s2,
                                        const uint8_t* s3, uint8_t* dst) {
  const int KB = l.K / 32;
  const long long total = static_cast<long long>(l.tiles) * KB * l.mt;
  const long long rec = static_cast<long long>(blockIdx.x) * 8 + threadIdx.x / 32;
  if (rec >= total)
    return;
  const int lane = threadIdx.x % 32, g = lane / 4, c = lane % 4;
  const int m = int(rec % l.mt);
  const long long tb = rec / l.mt;
  const int kb = int(tb % KB), t = int(tb / KB);
  int j = 0, row0 = 0;
  const bool valid = decode_mtile_source(l, t, m, j, row0);
  const uint8_t* src = j == 0 ? s0 : j == 1 ? s1 : j == 2 ? s2 : s3;
  uint8_t* out = dst + rec * kDecRecordBf16;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = row0 + g + 8 * h;
    uint4 v = make_uint4(0, 0, 0, 0);
    const size_t ld = l.src_ld[j] ? size_t(l.src_ld[j]) / 2 : size_t(l.K);
    if (valid && row < l.rows[j])
      v = *reinterpret_cast<const uint4*>(src + (size_t(row) * ld + kb * 32 + 8 * c) * 2);
    *reinterpret_cast<uint4*>(out + 512 * h + lane * 16) = v;
  }
}

__global__ void decode_pack_kernel(const DecodeLayout l, const uint8_t* s0,
                                   const uint8_t* s1, const uint8_t* s2,
                                   const uint8_t* s3, uint8_t* dst) {
  const int KB = l.K / 32;
  const long long total = static_cast<long long>(l.tiles) * KB * l.mt;
  const long long rec = static_cast<long long>(blockIdx.x) * 8 + threadIdx.x / 32;
  if (rec >= total)
    return;
  const int lane = threadIdx.x % 32, g = lane / 4, c = lane % 4;
  const int m = int(rec % l.mt);
  const long long tb = rec / l.mt;
  const int kb = int(tb % KB), t = int(tb / KB);
  int j = 0, row0 = 0;
  const bool valid = decode_mtile_source(l, t, m, j, row0);
  const uint8_t* src = j == 0 ? s0 : j == 1 ? s1 : j == 2 ? s2 : s3;
  const size_t row_bytes = l.src_ld[j] ? size_t(l.src_ld[j]) : size_t(KB) * 34;
  union {
    uint8_t b[16];
    uint4 v;
  } codes;
  uint32_t scales = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = row0 + g + 8 * h;
    const bool ok = valid && row < l.rows[j];
    const uint8_t* block = ok ? src + size_t(row) * row_bytes + size_t(kb) * 34 : nullptr;
    if (ok)
      scales |= uint32_t(block[0] | (block[1] << 8)) << (16 * h);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      codes.b[8 * h + i] = ok ? uint8_t(block[2 + 8 * c + i] ^ 0x80u) : 0x80u;
  }
  uint8_t* out = dst + rec * kDecRecord;
  *reinterpret_cast<uint4*>(out + lane * 16) = codes.v;
  if (c == 0)
    *reinterpret_cast<uint32_t*>(out + 512 + g * 4) = scales;
}

// Units of 32 blocks for one-m-tile tiles (17 KB) when K allows, else 16.
template <int kKind, int kMT>
cudaError_t launch_kind(const DecodeParams& p, int grid, cudaStream_t stream,
                        bool pdl) {
  // inputs of K <= kDecStagedK columns staged in shared memory: read once
  // per CTA, all chunks requested at once after the dependency wait, instead
  // of an L2 round trip per unit
  const bool staged = p.layout.K <= kDecStagedK && !p.layout.x_ld;
  auto kernel = staged ? decode_gemv_kernel<kKind, kMT, 16, true, false>
                       : decode_gemv_kernel<kKind, kMT, 16, false, false>;
  if constexpr (kMT == 1)
    if (p.layout.K % 1024 == 0)
      kernel = staged ? decode_gemv_kernel<kKind, kMT, 32, true, false>
                      : decode_gemv_kernel<kKind, kMT, 32, false, false>;
  if (p.layout.bf16) {
    // BF16 units: 16 blocks of one-m-tile tiles, else 8 (16-32 KB)
    if constexpr (kMT == 1)
      kernel = staged ? decode_gemv_kernel<kKind, kMT, 16, true, true>
                      : decode_gemv_kernel<kKind, kMT, 16, false, true>;
    else
      kernel = staged ? decode_gemv_kernel<kKind, kMT, 8, true, true>
                      : decode_gemv_kernel<kKind, kMT, 8, false, true>;
  }
  const int bytes = staged ? int(sizeof(DecodeSmem<true>))
                           : int(sizeof(DecodeSmem<false>));
  if (const cudaError_t e =
          ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), bytes))
    return e;
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(grid);
  config.blockDim = dim3(kDecThreads);
  config.dynamicSmemBytes = bytes;
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  config.attrs = attr;
  config.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelEx(&config, kernel, p);
}

}  // namespace

namespace {
// The m-tiles per tile (from `choices`, largest first) that minimise the
// most m-tiles any of `sms` CTAs holds when tiles go round-robin.
int pick_mtiles(int mtiles, int sms, std::initializer_list<int> choices) {
  int best = 0, best_load = 0;
  for (const int mt : choices) {
    const int tiles = (mtiles + mt - 1) / mt;
    const int load = (tiles + sms - 1) / sms * mt;
    if (!best || load < best_load) {
      best = mt;
      best_load = load;
    }
  }
  return best;
}
}  // namespace

bool decode_layout(DecodeLayout& l, int sms) {
  if (l.K <= 0 || l.K % 512 || sms <= 0)
    return false;
  if (l.kind == kDecPlain) {
    if (l.n_src < 1 || l.n_src > 4)
      return false;
    int mtiles = 0;
    for (int j = 0; j < l.n_src; ++j) {
      if (l.rows[j] <= 0)
        return false;
      l.first_mtile[j] = mtiles;
      mtiles += (l.rows[j] + 15) / 16;
    }
    l.first_mtile[l.n_src] = mtiles;
    l.mt = pick_mtiles(mtiles, sms, {4, 2, 1});
    l.tiles = (mtiles + l.mt - 1) / l.mt;
  } else if (l.kind == kDecSwiGLU) {
    if (l.n_src != 2 || l.rows[0] <= 0 || l.rows[0] != l.rows[1])
      return false;
    // m-tiles of gate + up rows, in pairs
    l.mt = 2 * pick_mtiles((l.rows[0] + 15) / 16, sms, {2, 1});
    l.tiles = (l.rows[0] + 8 * l.mt - 1) / (8 * l.mt);
  } else if (l.kind == kDecConv) {
    if (l.n_src != 1 || l.H <= 0 || l.H % 16 || l.rows[0] != 3 * l.H)
      return false;
    l.mt = 3;
    l.tiles = l.H / 16;
  } else {
    return false;
  }
  return l.tiles > 0;
}

size_t decode_packed_bytes(const DecodeLayout& l) {
  return size_t(l.tiles) * (l.K / 32) * l.mt *
         (l.bf16 ? kDecRecordBf16 : kDecRecord);
}

cudaError_t launch_decode_pack(const DecodeLayout& l,
                               const uint8_t* const src[4], uint8_t* dst,
                               cudaStream_t stream) {
  if (!dst || reinterpret_cast<uintptr_t>(dst) % 16 || l.tiles <= 0)
    return cudaErrorInvalidValue;
  for (int j = 0; j < (l.kind == kDecPlain ? l.n_src : l.kind == kDecSwiGLU ? 2 : 1); ++j)
    if (!src[j])
      return cudaErrorInvalidValue;
  const long long records =
      static_cast<long long>(l.tiles) * (l.K / 32) * l.mt;
  note_launch();
  if (l.bf16)
    decode_pack_bf16_kernel<<<unsigned((records + 7) / 8), 256, 0, stream>>>(
        l, src[0], src[1], src[2], src[3], dst);
  else
    decode_pack_kernel<<<unsigned((records + 7) / 8), 256, 0, stream>>>(
        l, src[0], src[1], src[2], src[3], dst);
  return cudaGetLastError();
}

int decode_grid(const DecodeLayout& l, int sms) {
  return std::min(sms, l.tiles);
}

cudaError_t launch_decode_gemv(const DecodeParams& p, int grid,
                               cudaStream_t stream, bool pdl) {
  const DecodeLayout& l = p.layout;
  if (grid <= 0 || grid > l.tiles || !p.w || !p.x || p.tokens < 1 ||
      p.tokens > kMaxBatch || l.K % 512 ||
      reinterpret_cast<uintptr_t>(p.x) % 16 ||
      reinterpret_cast<uintptr_t>(p.w) % 16)
    return cudaErrorInvalidValue;
  if (l.x_ld) {  // a K split: Plain, whole tiles per source, columns in range
    if (l.kind != kDecPlain || l.x_ld % 8)
      return cudaErrorInvalidValue;
    for (int j = 0; j < l.n_src; ++j)
      if (l.first_mtile[j] % l.mt || l.x_col[j] % 8 || l.x_col[j] < 0 ||
          l.x_col[j] + l.K > l.x_ld)
        return cudaErrorInvalidValue;
  }
  if (l.kind == kDecPlain) {
    for (int j = 0; j < l.n_src; ++j)
      if (!p.o[j].out)
        return cudaErrorInvalidValue;
    switch (l.mt) {
      case 1: return launch_kind<kDecPlain, 1>(p, grid, stream, pdl);
      case 2: return launch_kind<kDecPlain, 2>(p, grid, stream, pdl);
      case 4: return launch_kind<kDecPlain, 4>(p, grid, stream, pdl);
      default: return cudaErrorInvalidValue;
    }
  }
  if (l.kind == kDecSwiGLU) {
    if (!p.split_out && !p.f32_out)
      return cudaErrorInvalidValue;
    switch (l.mt) {
      case 2: return launch_kind<kDecSwiGLU, 2>(p, grid, stream, pdl);
      case 4: return launch_kind<kDecSwiGLU, 4>(p, grid, stream, pdl);
      default: return cudaErrorInvalidValue;
    }
  }
  if (l.kind == kDecConv) {
    if (!p.split_out || !p.conv_w || !p.rows || p.L < 2 || l.mt != 3)
      return cudaErrorInvalidValue;
    return launch_kind<kDecConv, 3>(p, grid, stream, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace lfm3
