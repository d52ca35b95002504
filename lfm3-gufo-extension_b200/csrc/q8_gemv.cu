// Q8_0 projections of up to eight FP32 rows; see q8_gemv.cuh.
//
// A tile is 16 rows of one weight (or 16 gate + 16 up rows, or the B, C and
// x rows of 16 channels) over all K columns, owned by one CTA from first
// load to epilogue: no split-K, no cross-CTA fix-up. K streams through a
// two-stage shared-memory ring in chunks (one TMA box per m-tile per chunk,
// ~35 KB), so the ring stays under half an SM and the next projection's CTA
// can start its copies while this one finishes (programmatic dependent
// launch). Eight consumer warps split each chunk's Q8 blocks and run them on
// the tensor cores:
//
//   A = a block's codes of 16 rows, decoded exactly to fp16
//   B = the input rows as two fp16 terms (hi, lo) of up to 8 tokens
//   C = sum over the block's 32 columns, FP32, then acc += d * C
//
// i.e. the reference's per-block order "sum += d * (sum of q * x)"
// (hip/ops.hip:784-809) with FP32 accumulation. Inside a block the 32
// columns are assigned to MMA k positions by a fixed permutation that the
// split-activation records follow, so every thread reads 8 contiguous codes.
// Warp partials merge through shared memory in warp order, so results never
// depend on timing.
#include "common.cuh"
#include "kernels.cuh"
#include "q8_gemv.cuh"
#include "tensor_map.hpp"

namespace lfm3 {

namespace {

constexpr int kMaxTileRows = 64;

struct GemvSmem {
  alignas(128) uint8_t ring[kGemvRingBytes];
  float red[kGemvWarps][kMaxTileRows * kMaxBatch];
  float tile[kMaxTileRows * kMaxBatch];
  uint64_t full[kGemvMaxSlots];
  uint64_t empty[kGemvMaxSlots];
};

template <int kMT, int kBlocks>
constexpr uint32_t stage_bytes() {
  return kMT * 16 * gemv_pitch_units(kBlocks) * 16;
}
// ring slots for a kind's chunks (each slot a multiple of 128 bytes)
template <int kMT, int kBlocks>
constexpr int ring_slots() {
  return kGemvRingBytes / stage_bytes<kMT, kBlocks>() < kGemvMaxSlots
             ? kGemvRingBytes / stage_bytes<kMT, kBlocks>()
             : kGemvMaxSlots;
}

// Issues the tiled copies of (tile t, chunk c) into dst (Plain: one box of
// the tile's 16 x kMT rows; otherwise one 16-row box per m-tile; boxes past
// the matrix are zero-filled and still count). The maps view each weight as
// [rows][row_bytes / 8] 8-byte elements, so a box row is one contiguous run
// of the chunk (plus its padding) and lands as one shared-memory row.
template <int kKind, int kBlocks, int kMT>
__device__ __forceinline__ void load_unit(const GemvParams& p, int t, int c,
                                          uint8_t* dst, uint64_t* bar) {
  constexpr int kBox = 16 * gemv_pitch_units(kBlocks) * 16;
  // chunk c starts at byte 34 * kBlocks * c of each row: in 8-byte
  // elements an even coordinate, so the copy starts 16-byte aligned
  const int x8 = c * (kBlocks * 34 / 8);
  if (kKind == kGemvPlain) {
    int j = 0;
#pragma unroll
    for (int q = 1; q < 4; ++q)
      if (q < p.n_out && t >= p.first_tile[q])
        j = q;
    tma_load_2d(dst, &p.maps[j], x8, (t - p.first_tile[j]) * 16 * kMT, bar);
  } else if (kKind == kGemvSwiGLU) {
    tma_load_2d(dst, &p.maps[0], x8, t * 16, bar);
    tma_load_2d(dst + kBox, &p.maps[1], x8, t * 16, bar);
  } else {
#pragma unroll
    for (int part = 0; part < 3; ++part)
      tma_load_2d(dst + part * kBox, &p.maps[0], x8, part * p.H + t * 16,
                  bar);
  }
}

// Codes of one block for rows g and g + 8 of an m-tile as the A fragments of
// the block's two k16 halves, plus the two rows' scales. `row` points at the
// block in row g; rows are `pitch` bytes apart.
template <bool kAligned>
__device__ __forceinline__ void block_fragments(const uint8_t* row, int pitch,
                                                int cq, uint32_t (&a1)[4],
                                                uint32_t (&a2)[4],
                                                float (&d)[2]) {
  uint32_t w[2][2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint8_t* r = row + h * 8 * pitch;
    d[h] = __half2float(*reinterpret_cast<const __half*>(r));
    if (kAligned) {
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(r + 2 + 8 * cq);
      w[h][0] = pw[0];
      w[h][1] = pw[1];
    } else {
      const uint32_t* pw = reinterpret_cast<const uint32_t*>(r + 8 * cq);
      const uint32_t v0 = pw[0], v1 = pw[1], v2 = pw[2];
      w[h][0] = __funnelshift_r(v0, v1, 16);
      w[h][1] = __funnelshift_r(v1, v2, 16);
    }
  }
  codes_to_half2(w[0][0], a1[0], a1[2]);
  codes_to_half2(w[1][0], a1[1], a1[3]);
  codes_to_half2(w[0][1], a2[0], a2[2]);
  codes_to_half2(w[1][1], a2[1], a2[3]);
}

// One block's contribution for every m-tile: 4 MMAs (two k16 halves x the
// hi and lo input terms), then acc += d * C.
template <bool kAligned, int kMT>
__device__ __forceinline__ void run_block(const uint8_t* block, int pitch,
                                          int cq, uint4 xh, uint4 xl,
                                          float (&acc)[kMT][4]) {
#pragma unroll
  for (int m = 0; m < kMT; ++m) {
    uint32_t a1[4], a2[4];
    float d[2];
    block_fragments<kAligned>(block + m * 16 * pitch, pitch, cq, a1, a2, d);
    // the hi and lo input terms in two independent MMA chains
    float ch[4] = {0, 0, 0, 0}, cl[4] = {0, 0, 0, 0};
    mma_f16(ch, a1, xh.x, xh.y);
    mma_f16(cl, a1, xl.x, xl.y);
    mma_f16(ch, a2, xh.z, xh.w);
    mma_f16(cl, a2, xl.z, xl.w);
    acc[m][0] = fmaf(d[0], ch[0] + cl[0], acc[m][0]);
    acc[m][1] = fmaf(d[0], ch[1] + cl[1], acc[m][1]);
    acc[m][2] = fmaf(d[1], ch[2] + cl[2], acc[m][2]);
    acc[m][3] = fmaf(d[1], ch[3] + cl[3], acc[m][3]);
  }
}

// Conv epilogue inputs of one (channel, token) read ahead of the step: the
// session's history window and the channel's taps.
constexpr int kConvAhead = 8;  // widths up to 8 are read ahead
struct ConvAhead {
  float hist[kConvAhead - 1], w[kConvAhead];
  bool ok;  // read for tile `blockIdx.x`
};
__device__ __forceinline__ ConvAhead conv_ahead(const GemvParams& p, int tid) {
  ConvAhead a;
  const int i = tid / kMaxBatch, tok = tid % kMaxBatch;
  const int ch = blockIdx.x * 16 + i, L = p.L;
  a.ok = i < 16 && tok < p.tokens && ch < p.H && L <= kConvAhead;
  if (a.ok) {
    const float* own = p.rows->layers[tok][p.layer].conv + size_t(ch) * (L - 1);
#pragma unroll
    for (int j = 0; j < kConvAhead - 1; ++j)
      a.hist[j] = j < L - 1 ? own[j] : 0.0F;
#pragma unroll
    for (int j = 0; j < kConvAhead; ++j)
      a.w[j] = j < L ? p.conv_w[size_t(ch) * L + j] : 0.0F;
  }
  return a;
}

template <int kKind, int kMT>
__device__ void gemv_epilogue(const GemvParams& p, const float* tile, int t,
                              int tid, const ConvAhead* ahead = nullptr) {
  if (kKind == kGemvPlain) {
    int j = 0;
#pragma unroll
    for (int q = 1; q < 4; ++q)
      if (q < p.n_out && t >= p.first_tile[q])
        j = q;
    for (int e = tid; e < kMT * 16 * kMaxBatch; e += kGemvWarps * 32) {
      const int i = e / kMaxBatch, tok = e % kMaxBatch;
      const int row = (t - p.first_tile[j]) * 16 * kMT + i;
      if (tok < p.tokens && row < p.o[j].rows)
        p.o[j].out[size_t(tok) * p.o[j].ld + row] = tile[e];
    }
    return;
  }
  const int i = tid / kMaxBatch, tok = tid % kMaxBatch;  // 16 rows x 8
  if (i >= 16 || tok >= p.tokens)
    return;
  if (kKind == kGemvSwiGLU) {
    const int row = t * 16 + i;
    if (row >= p.o[0].rows)
      return;
    const float g = tile[i * kMaxBatch + tok];
    const float u = tile[(16 + i) * kMaxBatch + tok];
    // BatchedSwiGLUActivationKernel's formula (hip/ops.hip:175-177)
    const float sig = 1.0F / (1.0F + expf(-g));
    const float h = (g * sig) * u;
    if (p.split_out)
      store_split(p.split_out, tok, p.split_width, row, h);
    if (p.o[0].out)
      p.o[0].out[size_t(tok) * p.o[0].ld + row] = h;
    return;
  }
  // Conv step per (channel, token), ConvolutionStep's expressions
  // (hip/ops.hip:1135-1151): FMA chain over the window oldest first, then
  // gate by C; the history shifts by one and keeps the newest B*x.
  const int ch = t * 16 + i;
  if (ch >= p.H)
    return;
  const int L = p.L;
  const float b = tile[i * kMaxBatch + tok];
  const float c = tile[(16 + i) * kMaxBatch + tok];
  const float x = tile[(32 + i) * kMaxBatch + tok];
  float* own = p.rows->layers[tok][p.layer].conv + size_t(ch) * (L - 1);
  const float current = b * x;
  float sum = 0;
  if (ahead && ahead->ok && t == int(blockIdx.x)) {
#pragma unroll
    for (int j = 0; j < kConvAhead - 1; ++j)
      if (j < L - 1)
        sum = fmaf(ahead->w[j], ahead->hist[j], sum);
    sum = fmaf(ahead->w[L - 1], current, sum);
#pragma unroll
    for (int j = 0; j < kConvAhead - 2; ++j)
      if (j < L - 2)
        own[j] = ahead->hist[j + 1];
  } else {
    const float* w = p.conv_w + size_t(ch) * L;
    for (int j = 0; j < L - 1; ++j)
      sum = fmaf(w[j], own[j], sum);
    sum = fmaf(w[L - 1], current, sum);
    for (int j = 0; j < L - 2; ++j)
      own[j] = own[j + 1];
  }
  own[L - 2] = current;
  store_split(p.split_out, tok, p.split_width, ch, sum * c);
}

template <int kKind, int kBlocks, int kMT>
__device__ void gemv_body(const GemvParams& p, GemvSmem& s) {
  constexpr int kPitch = gemv_pitch_units(kBlocks) * 16;
  constexpr uint32_t kStageBytes = stage_bytes<kMT, kBlocks>();
  constexpr int kSlots = ring_slots<kMT, kBlocks>();
  static_assert(kSlots >= 2 && kStageBytes % 128 == 0, "ring slots");
  constexpr int kPerWarp = kBlocks / kGemvWarps;  // even: 8, 4 or 2
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int grid = gridDim.x, chunks = p.chunks;

  if (warp == kGemvWarps) {
    // ---- producer: weights only, so it may run ahead of the previous
    // kernel in the stream
    if (lane != 0)
      return;
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < p.tiles; t += grid)
      for (int c = 0; c < chunks; ++c) {
        if (!mbar_wait(&s.empty[stage], phase ^ 1, kErrGemvEmptyWait))
          return;
        mbar_arrive_expect_tx(&s.full[stage], kStageBytes);
        load_unit<kKind, kBlocks, kMT>(p, t, c, s.ring + stage * kStageBytes,
                                       &s.full[stage]);
        if (++stage == kSlots) {
          stage = 0;
          phase ^= 1;
        }
      }
    return;
  }

  // ---- consumers
  // the conv step's history and taps of the first tile: written only by
  // this layer's step of an earlier round, so read before the wait
  ConvAhead ahead{};
  if (kKind == kGemvConv)
    ahead = conv_ahead(p, tid);
  grid_dependency_wait();
  const int g = lane / 4, cq = lane % 4;
  const uint4* x = static_cast<const uint4*>(p.x);
  const int records = p.K / 8;
  const bool token_live = g < p.tokens;
  // input terms (hi, lo) of token g for global block kb
  const auto fetch_x = [&](int kb, uint4& hi, uint4& lo) {
    hi = make_uint4(0, 0, 0, 0);
    lo = hi;
    if (token_live) {
      const uint4* rec = x + (size_t(g) * records + kb * 4 + cq) * 2;
      hi = __ldg(rec);
      lo = __ldg(rec + 1);
    }
  };
  int stage = 0;
  uint32_t phase = 0;
  const int b0 = warp * kPerWarp;  // this warp's first block in each chunk
  // the input terms of this warp's blocks of one chunk
  struct ChunkX {
    uint4 h[kPerWarp], l[kPerWarp];
  };
  const auto fetch_chunk = [&](int c, ChunkX& x) {
#pragma unroll
    for (int i = 0; i < kPerWarp; ++i)
      fetch_x(c * kBlocks + b0 + i, x.h[i], x.l[i]);
  };
  for (int t = blockIdx.x; t < p.tiles; t += grid) {
    float acc[kMT][4];
#pragma unroll
    for (int m = 0; m < kMT; ++m)
#pragma unroll
      for (int j = 0; j < 4; ++j)
        acc[m][j] = 0;
    // every input load of a chunk in flight at once, the next chunk's
    // issued before this one's math
    ChunkX cur, next;
    fetch_chunk(0, cur);
    for (int c = 0; c < chunks; ++c) {
      if (c + 1 < chunks)
        fetch_chunk(c + 1, next);
      if (!mbar_wait(&s.full[stage], phase, kErrGemvFullWait))
        return;
      const uint8_t* rows = s.ring + stage * kStageBytes + g * kPitch;
#pragma unroll
      for (int pair = 0; pair < kPerWarp / 2; ++pair) {
        const int b = b0 + 2 * pair;
        // block b starts two bytes into a word (b even), b + 1 on a word
        run_block<false, kMT>(rows + b * 34, kPitch, cq, cur.h[2 * pair],
                              cur.l[2 * pair], acc);
        run_block<true, kMT>(rows + (b + 1) * 34, kPitch, cq,
                             cur.h[2 * pair + 1], cur.l[2 * pair + 1], acc);
      }
      cur = next;
      __syncwarp();
      if (lane == 0)
        mbar_arrive(&s.empty[stage]);
      if (++stage == kSlots) {
        stage = 0;
        phase ^= 1;
      }
    }
    // ---- tile t complete: merge the warps in order, then the epilogue
    float* red = s.red[warp];
#pragma unroll
    for (int m = 0; m < kMT; ++m) {
      const int r = m * 16 + g;
      red[r * kMaxBatch + 2 * cq] = acc[m][0];
      red[r * kMaxBatch + 2 * cq + 1] = acc[m][1];
      red[(r + 8) * kMaxBatch + 2 * cq] = acc[m][2];
      red[(r + 8) * kMaxBatch + 2 * cq + 1] = acc[m][3];
    }
    named_barrier(1, kGemvWarps * 32);
    for (int e = tid; e < kMT * 16 * kMaxBatch; e += kGemvWarps * 32) {
      float v = s.red[0][e];
#pragma unroll
      for (int q = 1; q < kGemvWarps; ++q)
        v += s.red[q][e];
      s.tile[e] = v;
    }
    named_barrier(1, kGemvWarps * 32);
    gemv_epilogue<kKind, kMT>(p, s.tile, t, tid, &ahead);
  }
}

__global__ void __launch_bounds__(kGemvThreads, 1)
    q8_gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  GemvSmem& s = *reinterpret_cast<GemvSmem*>(smem_raw);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kGemvMaxSlots; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], kGemvWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  allow_dependents();
  if (p.kind == kGemvPlain) {
    if (p.wide)
      gemv_body<kGemvPlain, 16, 4>(p, s);
    else if (p.chunk_blocks == 32)
      gemv_body<kGemvPlain, 32, 1>(p, s);
    else
      gemv_body<kGemvPlain, 16, 1>(p, s);
  } else if (p.kind == kGemvSwiGLU) {
    if (p.chunk_blocks == 32)
      gemv_body<kGemvSwiGLU, 32, 2>(p, s);
    else
      gemv_body<kGemvSwiGLU, 16, 2>(p, s);
  } else {
    gemv_body<kGemvConv, 16, 3>(p, s);
  }
}

// ---- BF16 projections -------------------------------------------------------
constexpr int kBf16Chunk = 1024;  // K columns of the input staged per pass
constexpr int kBf16Threads = 256;

struct Bf16Smem {
  float x[kMaxBatch][kBf16Chunk + 4];
  float tile[kMaxTileRows * kMaxBatch];
};

// Weight row of tile row r of tile t (BF16, K elements), or null past the
// matrix.
template <int kKind, int kMT>
__device__ __forceinline__ const uint16_t* bf16_row(const GemvParams& p, int t,
                                                    int r) {
  int matrix = 0, row = 0;
  if (kKind == kGemvPlain) {
#pragma unroll
    for (int q = 1; q < 4; ++q)
      if (q < p.n_out && t >= p.first_tile[q])
        matrix = q;
    row = (t - p.first_tile[matrix]) * 16 * kMT + r;
  } else if (kKind == kGemvSwiGLU) {
    matrix = r / 16;
    row = t * 16 + r % 16;
  } else {
    row = (r / 16) * p.H + t * 16 + r % 16;
    if (t * 16 + r % 16 >= p.H)
      return nullptr;
  }
  if (row >= p.o[matrix].rows)
    return nullptr;
  return reinterpret_cast<const uint16_t*>(p.o[matrix].w) + size_t(row) * p.K;
}

__device__ __forceinline__ void bf16x8(const uint4& w, float (&f)[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
  }
}

template <int kKind, int kMT>
__global__ void __launch_bounds__(kBf16Threads)
    bf16_gemv_kernel(const __grid_constant__ GemvParams p, const float* x32,
                     int x_ld, int rows) {
  constexpr int kRows = 16 * kMT, kR = kRows / 8;  // tile rows, rows per warp
  __shared__ Bf16Smem s;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int t = blockIdx.x;
  const int t0 = blockIdx.y * kMaxBatch;  // first input row of this group
  const int nt = x32 ? min(kMaxBatch, rows - t0) : p.tokens;
  grid_dependency_wait();
  const uint16_t* w[kR];
#pragma unroll
  for (int r = 0; r < kR; ++r)
    w[r] = bf16_row<kKind, kMT>(p, t, warp * kR + r);
  float acc[kR][kMaxBatch];
#pragma unroll
  for (int r = 0; r < kR; ++r)
#pragma unroll
    for (int j = 0; j < kMaxBatch; ++j)
      acc[r][j] = 0;
  // columns per staging pass: the largest of 1024, 512, 256 dividing K
  const int chunk = p.K % 1024 == 0 ? 1024 : p.K % 512 == 0 ? 512 : 256;
  for (int c0 = 0; c0 < p.K; c0 += chunk) {
    __syncthreads();
    // stage the input rows' columns c0 .. c0 + chunk - 1 as FP32 (8 per
    // thread-step: one split record, or two float4)
    for (int e = tid; e < kMaxBatch * chunk / 8; e += kBf16Threads) {
      const int tok = e / (chunk / 8), k = (e % (chunk / 8)) * 8;
      float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (tok < nt) {
        if (x32) {
          const float* src = x32 + size_t(t0 + tok) * x_ld + c0 + k;
          const float4 a = *reinterpret_cast<const float4*>(src);
          const float4 b = *reinterpret_cast<const float4*>(src + 4);
          v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w;
          v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
        } else {
          const uint4* rec = static_cast<const uint4*>(p.x) +
                             (size_t(tok) * (p.K / 8) + (c0 + k) / 8) * 2;
          const uint4 hi = rec[0], lo = rec[1];
          const uint32_t h[4] = {hi.x, hi.y, hi.z, hi.w};
          const uint32_t l[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&l[i]));
            v[2 * i] = a.x + b.x;
            v[2 * i + 1] = a.y + b.y;
          }
        }
      }
      float* dst = &s.x[tok][k];
      *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
    __syncthreads();
    for (int k = lane * 8; k < chunk; k += 256) {
      float wf[kR][8];
#pragma unroll
      for (int r = 0; r < kR; ++r) {
        uint4 raw = make_uint4(0, 0, 0, 0);
        if (w[r])
          raw = __ldg(reinterpret_cast<const uint4*>(w[r] + c0 + k));
        bf16x8(raw, wf[r]);
      }
#pragma unroll
      for (int tok = 0; tok < kMaxBatch; ++tok) {
        const float4 a = *reinterpret_cast<const float4*>(&s.x[tok][k]);
        const float4 b = *reinterpret_cast<const float4*>(&s.x[tok][k + 4]);
        const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int r = 0; r < kR; ++r)
#pragma unroll
          for (int i = 0; i < 8; ++i)
            acc[r][tok] = fmaf(wf[r][i], xv[i], acc[r][tok]);
      }
    }
  }
  allow_dependents();
  // lanes' partial sums in a fixed butterfly order
#pragma unroll
  for (int r = 0; r < kR; ++r)
#pragma unroll
    for (int tok = 0; tok < kMaxBatch; ++tok) {
      const float v = warp_sum(acc[r][tok]);
      if (lane == 0)
        s.tile[(warp * kR + r) * kMaxBatch + tok] = v;
    }
  __syncthreads();
  if (!x32) {
    gemv_epilogue<kKind, kMT>(p, s.tile, t, tid);
    return;
  }
  // prompt rows t0 .. t0 + nt - 1
  for (int e = tid; e < 16 * kMaxBatch * (kKind == kGemvPlain ? kMT : 1);
       e += kBf16Threads) {
    const int i = e / kMaxBatch, tok = e % kMaxBatch;
    if (tok >= nt)
      continue;
    if (kKind == kGemvPlain) {
      int j = 0;
#pragma unroll
      for (int q = 1; q < 4; ++q)
        if (q < p.n_out && t >= p.first_tile[q])
          j = q;
      const int row = (t - p.first_tile[j]) * 16 * kMT + i;
      if (row < p.o[j].rows)
        p.o[j].out[size_t(t0 + tok) * p.o[j].ld + row] = s.tile[e];
    } else {
      const int row = t * 16 + i;
      if (row >= p.o[0].rows)
        continue;
      const float g = s.tile[i * kMaxBatch + tok];
      const float u = s.tile[(16 + i) * kMaxBatch + tok];
      // BatchedSwiGLUActivationKernel's formula (hip/ops.hip:175-177)
      const float sig = 1.0F / (1.0F + expf(-g));
      p.o[0].out[size_t(t0 + tok) * p.o[0].ld + row] = (g * sig) * u;
    }
  }
}

}  // namespace

bool gemv_plan(GemvParams& p, int sms) {
  if (p.K <= 0 || p.K % 512)
    return false;
  p.wide = 0;
  if (p.kind == kGemvPlain) {
    int wide_tiles = 0;
    for (int j = 0; j < p.n_out; ++j)
      wide_tiles += (p.o[j].rows + 63) / 64;
    // two or more 64-row tiles for each of the 2 x sms CTA slots
    p.wide = wide_tiles >= 4 * sms;
    p.chunk_blocks = p.wide ? 16 : p.K % 1024 == 0 ? 32 : 16;
  } else if (p.kind == kGemvSwiGLU) {
    p.chunk_blocks = p.K % 1024 == 0 ? 32 : 16;
  } else {
    p.chunk_blocks = 16;
  }
  p.chunks = p.K / (32 * p.chunk_blocks);
  if (p.kind == kGemvPlain) {
    int tiles = 0;
    const int rows = p.wide ? 64 : 16;
    for (int j = 0; j < p.n_out; ++j) {
      p.first_tile[j] = tiles;
      tiles += (p.o[j].rows + rows - 1) / rows;
    }
    p.first_tile[p.n_out] = tiles;
    p.tiles = tiles;
  } else if (p.kind == kGemvSwiGLU) {
    p.tiles = (p.o[0].rows + 15) / 16;
  } else {
    if (p.H % 16)
      return false;
    p.tiles = p.H / 16;
  }
  return p.tiles > 0;
}

int gemv_grid(int tiles, int sms) {
  // One CTA per SM (registers for every input load of two chunks in flight)
  // leaves room for the next kernel's CTA, whose producer then streams that
  // projection's weights while this one finishes (programmatic dependent
  // launch).
  return tiles < sms ? tiles : sms;
}

int gemv_box_rows(const GemvParams& p) {
  return p.kind == kGemvPlain && p.wide ? 64 : 16;
}

cudaError_t fill_gemv_maps(GemvParams& p) {
  const size_t row_bytes = size_t(p.K / 32) * 34;
  const int outputs =
      p.kind == kGemvPlain ? p.n_out : p.kind == kGemvSwiGLU ? 2 : 1;
  for (int j = 0; j < outputs; ++j) {
    const cudaError_t e =
        encode_q8_rows(&p.maps[j], p.o[j].w, row_bytes, p.o[j].rows,
                       gemv_pitch_units(p.chunk_blocks) * 16,
                       gemv_box_rows(p));
    if (e != cudaSuccess)
      return e;
  }
  return cudaSuccess;
}

bool bf16_plan(GemvParams& p) {
  if (p.K <= 0 || p.K % 256)
    return false;
  p.wide = 0;
  p.chunk_blocks = 0;
  p.chunks = 0;
  if (p.kind == kGemvPlain) {
    int tiles = 0;
    for (int j = 0; j < p.n_out; ++j) {
      p.first_tile[j] = tiles;
      tiles += (p.o[j].rows + 15) / 16;
    }
    p.first_tile[p.n_out] = tiles;
    p.tiles = tiles;
  } else if (p.kind == kGemvSwiGLU) {
    p.tiles = (p.o[0].rows + 15) / 16;
  } else {
    if (p.H % 16)
      return false;
    p.tiles = p.H / 16;
  }
  return p.tiles > 0;
}

cudaError_t launch_bf16_gemv(const GemvParams& p, const float* x32, int x_ld,
                             int rows, cudaStream_t stream) {
  if (p.tiles <= 0 || (x32 && (rows <= 0 || p.kind == kGemvConv ||
                               x_ld % 4 || x_ld < p.K)) ||
      (!x32 && (!p.x || p.tokens < 1 || p.tokens > kMaxBatch)))
    return cudaErrorInvalidValue;
  const dim3 grid(p.tiles, x32 ? (rows + kMaxBatch - 1) / kMaxBatch : 1);
  note_launch();
  if (p.kind == kGemvPlain)
    bf16_gemv_kernel<kGemvPlain, 1>
        <<<grid, kBf16Threads, 0, stream>>>(p, x32, x_ld, rows);
  else if (p.kind == kGemvSwiGLU)
    bf16_gemv_kernel<kGemvSwiGLU, 2>
        <<<grid, kBf16Threads, 0, stream>>>(p, x32, x_ld, rows);
  else
    bf16_gemv_kernel<kGemvConv, 3>
        <<<grid, kBf16Threads, 0, stream>>>(p, x32, x_ld, rows);
  return cudaGetLastError();
}

cudaError_t launch_q8_gemv(const GemvParams& p, int grid, cudaStream_t stream,
                           bool pdl) {
  if (const cudaError_t e = ensure_dynamic_smem(
          reinterpret_cast<const void*>(q8_gemv_kernel), int(sizeof(GemvSmem))))
    return e;
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(grid);
  config.blockDim = dim3(kGemvThreads);
  config.dynamicSmemBytes = sizeof(GemvSmem);
  config.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  config.attrs = attr;
  config.numAttrs = 1;
  note_launch();
  return cudaLaunchKernelEx(&config, q8_gemv_kernel, p);
}

}  // namespace lfm3
