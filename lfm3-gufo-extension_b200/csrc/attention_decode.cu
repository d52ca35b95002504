// Decode attention for every row of a round in one launch.
//
// Grid (kv_heads, splits, rows): a CTA owns one KV group of one row and a
// span of that row's keys, so ragged depths need no per-row launches. Every
// CTA normalises and rotates its group's query heads itself (cheap), and the
// CTA whose span ends at the row's position also stores the new K/V row in
// the ring. Keys stream through shared memory in tiles of 64 and an online
// softmax keeps FP32 scores, probabilities and accumulators (the decode
// precision of hip/ops.hip:1562-1691). Both products run on the tensor cores
// (mma.sync m16n8k16, FP32 accumulation) with the FP32 operands split in two
// fp16 terms, x = hi + lo (22 significant bits): S^T = K (Q_hi + Q_lo)^T with
// the keys as M and the group's heads (padded to 8) as N, then
// O^T = V^T (P_hi + P_lo)^T with the 128 dimensions as M; K and V are the
// cache's fp16 values, exactly. With several spans, each CTA writes its
// maximum, denominator and unnormalised output, and whichever CTA of the
// group finishes last (a ticket, not a wait) merges them in span order and
// applies the gate (hip/ops.hip:1710-1728).
#include "attention.cuh"
#include "common.cuh"
#include "kernels.cuh"

namespace lfm3 {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr float kScoreScale = 0.0883883476483184405F;  // 1 / sqrt(128)

// Shared rows are 16-byte pieces of 8 fp16; piece c of row i sits at
// c ^ (i & 7), so the eight rows of one ldmatrix fetch hit distinct banks.
__device__ __forceinline__ int at128(int row, int piece) {  // 128-wide rows
  return row * kHeadDim + ((piece ^ (row & 7)) << 3);
}
__device__ __forceinline__ int at64(int row, int piece) {  // 64-wide rows
  return row * kDecodeTile + ((piece ^ (row & 7)) << 3);
}

// Two key tiles in flight: K and V of tile t in buffer t % 2.
constexpr int kTileBufs = 2;
struct DecodeSmem {
  alignas(16) __half k[kTileBufs][kDecodeTile * kHeadDim];  // [key][dim]
  alignas(16) __half v[kTileBufs][kDecodeTile * kHeadDim];  // [key][dim]
  alignas(16) __half qh[8 * kHeadDim], ql[8 * kHeadDim];      // [head][dim]
  alignas(16) __half ph[8 * kDecodeTile], pl[8 * kDecodeTile];  // [head][key]
  float tile_max[kWarps][8];
  float l[kWarps][8];  // running denominators of each warp's keys
  float m[8], lsum[8];
  alignas(16) __half newk[kHeadDim], newv[kHeadDim];  // the row at `position`
  int last;
};
// After the key loop the first K tile holds the output and the merge
// weights.
static_assert(sizeof(float) * (8 * kHeadDim + 2 * 8 * kMaxDecodeSplits) <=
                  sizeof(__half) * kDecodeTile * kHeadDim,
              "output staging fits the K tile");

// 16 bytes global -> shared, zero-filled when !valid (cp.async, L1 bypassed)
__device__ __forceinline__ void cp_async16(void* dst, const void* src,
                                           bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// every group but the newest has landed (this thread's copies)
__device__ __forceinline__ void cp_async_wait_older() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile(
      "ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
      : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_addr(p)));
}

// A lane's share of one 128-wide head: pairs (i, i + 64) for
// i in {lane, lane + 32}. The norm weights and the rotation of the row's
// position are constants of the launch, read before the dependency wait.
struct LaneNorm {
  float a[2], b[2];  // w[i], w[i + 64]
};
struct LaneRotation {
  float cs[2], sn[2];
};
__device__ __forceinline__ LaneNorm lane_norm(const float* w, int lane) {
  LaneNorm n;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    n.a[j] = w[lane + 32 * j];
    n.b[j] = w[lane + 32 * j + 64];
  }
  return n;
}
__device__ __forceinline__ LaneRotation lane_rotation(const float* freq,
                                                      const float* factors,
                                                      int position, int lane) {
  LaneRotation t;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = lane + 32 * j;
    float angle = float(position) * freq[i];
    if (factors)
      angle /= factors[i];
    sincosf(angle, &t.sn[j], &t.cs[j]);
  }
  return t;
}
// RMSNorm and RoPE of the head held as the lane's pairs; returns the
// rotated pairs.
__device__ __forceinline__ void norm_rope(float (&x0)[2], float (&x1)[2],
                                          const LaneNorm& w,
                                          const LaneRotation& t, float eps) {
  float squares = 0;
#pragma unroll
  for (int j = 0; j < 2; ++j)
    squares += x0[j] * x0[j] + x1[j] * x1[j];
  const float inv = 1.0F / sqrtf(warp_sum(squares) / 128.0F + eps);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const float a = (x0[j] * inv) * w.a[j], b = (x1[j] * inv) * w.b[j];
    x0[j] = a * t.cs[j] - b * t.sn[j];
    x1[j] = b * t.cs[j] + a * t.sn[j];
  }
}

// Four CTAs per SM (128 registers): a round's spans run in one wave.
template <int G>
__global__ void __launch_bounds__(kThreads, 3)
    decode_attention_kernel(const __grid_constant__ DecodeAttentionParams p) {
  extern __shared__ __align__(128) uint8_t decode_smem_raw[];
  DecodeSmem& s = *reinterpret_cast<DecodeSmem*>(decode_smem_raw);
  const int g = blockIdx.x, split = blockIdx.y, r = blockIdx.z;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  // ---- before the dependency wait: the row table (written before the
  // round), the launch's constants and, with settled rings, the first key
  // tile
  const bool op = p.rows == nullptr;
  const int position = op ? p.position : p.rows->position[r];
  const LayerState state =
      op ? LayerState{nullptr, const_cast<__half*>(p.ring_k),
                      const_cast<__half*>(p.ring_v), p.capacity, 0}
         : p.rows->layers[r][p.layer];
  const int capacity = state.capacity;
  const int first = p.window > 0 ? max(0, position + 1 - p.window) : 0;
  const int tiles = (position + 1 - first + kDecodeTile - 1) / kDecodeTile;
  const int per = decode_span_tiles(tiles, p.max_splits, p.span_tiles);
  const int used = (tiles + per - 1) / per;  // decode_spans_used
  if (split >= used)
    return;
  const int begin = first + split * per * kDecodeTile;
  const int end = min(begin + per * kDecodeTile, position + 1);
  const size_t stride = size_t(p.kv_heads) * kHeadDim;
  // this CTA writes the row at `position` (and uses it from shared memory)
  const bool stores_row = !op && split == used - 1;
  LaneNorm qn{}, kn{};
  LaneRotation rot{};
  if (!op) {
    qn = lane_norm(p.q_norm, lane);
    kn = lane_norm(p.k_norm, lane);
    rot = lane_rotation(p.freq, p.factors, position, lane);
  }

  // ---- K and V rows of a tile (16-byte pieces) copied into buffer
  // (tile % kTileBufs), one cp.async group per tile (empty past the span)
  constexpr int kPieces = kDecodeTile * 16 / kThreads;
  const auto issue_tile = [&](int tile) {
    const int base = begin + tile * kDecodeTile;
    if (base < end) {
      const int n = min(kDecodeTile, end - base);
      const int slot0 = base % capacity;  // ring slot of key `base`
      __half* sk = s.k[tile % kTileBufs];
      __half* sv = s.v[tile % kTileBufs];
#pragma unroll
      for (int j = 0; j < kPieces; ++j) {
        const int c = tid + j * kThreads, key = c / 16, piece = c % 16;
        const int t = base + min(key, n - 1);
        const __half *ks = state.k, *vs = state.v;
        int slot = slot0 + min(key, n - 1);
        if (slot >= capacity)
          slot = capacity >= kDecodeTile ? slot - capacity : slot % capacity;
        size_t row = size_t(slot) * stride;
        if (op && t >= position) {
          ks = p.chunk_k;
          vs = p.chunk_v;
          row = size_t(t - position) * stride;
        }
        row += size_t(g) * kHeadDim;
        cp_async16(&sk[at128(key, piece)],
                   reinterpret_cast<const uint4*>(ks + row) + piece, key < n);
        cp_async16(&sv[at128(key, piece)],
                   reinterpret_cast<const uint4*>(vs + row) + piece, key < n);
      }
    }
    cp_async_commit();
  };
  // with settled rings the first tiles are copied while the previous
  // kernel finishes (the row at `position` is patched in below)
  const bool early = !op && p.ring_settled;
  if (early) {
    issue_tile(0);
    issue_tile(1);
  }
  grid_dependency_wait();
  allow_dependents();
  if (!early) {
    issue_tile(0);
    issue_tile(1);
  }

  // ---- query heads of this group (normalised, rotated), as hi + lo fp16
  // terms; heads G..7 are zero
  for (int h = warp; h < 8; h += kWarps) {
    float x0[2] = {0, 0}, x1[2] = {0, 0};
    if (h < G) {
      const float* qr =
          p.q + size_t(r) * p.ldq + size_t(g * G + h) * kHeadDim;
      x0[0] = qr[lane], x0[1] = qr[lane + 32];
      x1[0] = qr[lane + 64], x1[1] = qr[lane + 96];
      if (!op)
        norm_rope(x0, x1, qn, rot, p.eps);
    }
    const float e[4] = {x0[0], x0[1], x1[0], x1[1]};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = lane + 32 * j;
      const SplitPair t = split_value(e[j]);
      s.qh[at128(h, i / 8) + i % 8] = t.hi;
      s.ql[at128(h, i / 8) + i % 8] = t.lo;
    }
  }
  // ---- the new K/V row goes to its ring slot (span holding `position`)
  if (stores_row && warp == 0) {
    const float* kx = p.k + size_t(r) * p.ldk + size_t(g) * kHeadDim;
    const float* vx = p.v + size_t(r) * p.ldk + size_t(g) * kHeadDim;
    float x0[2] = {kx[lane], kx[lane + 32]};
    float x1[2] = {kx[lane + 64], kx[lane + 96]};
    norm_rope(x0, x1, kn, rot, p.eps);
    const size_t slot = size_t(position % capacity) * stride +
                        size_t(g) * kHeadDim;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = lane + 32 * j;
      const __half k0 = __float2half_rn(x0[j]), k1 = __float2half_rn(x1[j]);
      const __half v0 = __float2half_rn(vx[i]), v1 = __float2half_rn(vx[i + 64]);
      state.k[slot + i] = k0;
      state.k[slot + i + 64] = k1;
      state.v[slot + i] = v0;
      state.v[slot + i + 64] = v1;
      s.newk[i] = k0;
      s.newk[i + 64] = k1;
      s.newv[i] = v0;
      s.newv[i + 64] = v1;
    }
  }
  if (tid < kWarps * 8)
    s.l[tid / 8][tid % 8] = 0;
  __syncthreads();

  // fragment coordinates: row fg (and fg + 8), column pair 2 cq, 2 cq + 1
  const int fg = lane / 4, cq = lane % 4;
  // ldmatrix lane roles: matrix mj = lane / 8 takes its row from lane mrow
  const int mj = lane / 8, mrow = lane % 8;
  // this thread's running maxima of heads 2 cq, 2 cq + 1 (every thread holds
  // the same values) and its O^T fragments of dimension tiles 2 w, 2 w + 1
  float mrun[2] = {-INFINITY, -INFINITY};
  float o[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};

  for (int tile = 0, base = begin; base < end; ++tile, base += kDecodeTile) {
    const int n = min(kDecodeTile, end - base);
    __half* const tk = s.k[tile % kTileBufs];
    __half* const tv = s.v[tile % kTileBufs];
    cp_async_wait_older();  // this tile's group (the next one may fly)
    __syncthreads();
    if (stores_row && position >= base && position < base + n) {
      // the ring slot may have been copied before this CTA wrote it
      if (tid < 32) {
        const int key = position - base;
        for (int piece = tid % 16; piece < 16; piece += 16) {
          if (tid < 16)
            *reinterpret_cast<uint4*>(&tk[at128(key, piece)]) =
                *reinterpret_cast<const uint4*>(&s.newk[piece * 8]);
          else
            *reinterpret_cast<uint4*>(&tv[at128(key, piece)]) =
                *reinterpret_cast<const uint4*>(&s.newv[piece * 8]);
        }
      }
      __syncthreads();
    }

    // ---- S^T = K Q^T: warp w owns keys 16 w .. 16 w + 15
    float sh[4] = {0, 0, 0, 0}, sl[4] = {0, 0, 0, 0};
    {
      const int key = warp * 16 + (mj & 1) * 8 + mrow;
#pragma unroll
      for (int ks = 0; ks < kHeadDim / 16; ++ks) {
        uint32_t a[4], bh[2], bl[2];
        ldsm_x4(a, &tk[at128(key, 2 * ks + (mj >> 1))]);
        ldsm_x2(bh, &s.qh[at128(mrow, 2 * ks + (mj & 1))]);
        ldsm_x2(bl, &s.ql[at128(mrow, 2 * ks + (mj & 1))]);
        mma_f16(sh, a, bh[0], bh[1]);
        mma_f16(sl, a, bl[0], bl[1]);
      }
    }
    // this thread: keys k0 = 16 w + fg and k0 + 8, heads 2 cq and 2 cq + 1
    const int k0 = warp * 16 + fg;
    float sc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      sc[i] = (sh[i] + sl[i]) * kScoreScale;
    if (k0 >= n)
      sc[0] = sc[1] = -INFINITY;
    if (k0 + 8 >= n)
      sc[2] = sc[3] = -INFINITY;
    float t0 = fmaxf(sc[0], sc[2]), t1 = fmaxf(sc[1], sc[3]);
#pragma unroll
    for (int x = 4; x < 32; x <<= 1) {
      t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, x));
      t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, x));
    }
    if (fg == 0) {
      s.tile_max[warp][2 * cq] = t0;
      s.tile_max[warp][2 * cq + 1] = t1;
    }
    __syncthreads();
    // ---- online softmax over the tile's keys of every warp
    float top[2] = {s.tile_max[0][2 * cq], s.tile_max[0][2 * cq + 1]};
#pragma unroll
    for (int w = 1; w < kWarps; ++w) {
      top[0] = fmaxf(top[0], s.tile_max[w][2 * cq]);
      top[1] = fmaxf(top[1], s.tile_max[w][2 * cq + 1]);
    }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float next = fmaxf(mrun[h], top[h]);
      alpha[h] = expf(mrun[h] - next);  // 0 for the first tile
      mrun[h] = next;
    }
    const float pr[4] = {expf(sc[0] - mrun[0]), expf(sc[1] - mrun[1]),
                         expf(sc[2] - mrun[0]), expf(sc[3] - mrun[1])};
    float q0 = pr[0] + pr[2], q1 = pr[1] + pr[3];
#pragma unroll
    for (int x = 4; x < 32; x <<= 1) {
      q0 += __shfl_xor_sync(0xffffffffu, q0, x);
      q1 += __shfl_xor_sync(0xffffffffu, q1, x);
    }
    if (fg == 0) {
      s.l[warp][2 * cq] = s.l[warp][2 * cq] * alpha[0] + q0;
      s.l[warp][2 * cq + 1] = s.l[warp][2 * cq + 1] * alpha[1] + q1;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int head = 2 * cq + (i & 1), key = k0 + (i >> 1) * 8;
      const SplitPair t = split_value(pr[i]);
      s.ph[at64(head, key / 8) + key % 8] = t.hi;
      s.pl[at64(head, key / 8) + key % 8] = t.lo;
    }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      o[mt][0] *= alpha[0];
      o[mt][1] *= alpha[1];
      o[mt][2] *= alpha[0];
      o[mt][3] *= alpha[1];
    }
    __syncthreads();
    // ---- O^T += V^T P^T: warp w owns dimensions 32 w .. 32 w + 31
#pragma unroll
    for (int ks = 0; ks < kDecodeTile / 16; ++ks) {
      uint32_t bh[2], bl[2];
      ldsm_x2(bh, &s.ph[at64(mrow, 2 * ks + (mj & 1))]);
      ldsm_x2(bl, &s.pl[at64(mrow, 2 * ks + (mj & 1))]);
      const int key = ks * 16 + (mj >> 1) * 8 + mrow;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t a[4];
        ldsm_x4_trans(a, &tv[at128(key, 2 * (2 * warp + mt) + (mj & 1))]);
        mma_f16(o[mt], a, bh[0], bh[1]);
        mma_f16(o[mt], a, bl[0], bl[1]);
      }
    }
    __syncthreads();  // this tile's buffers and p are free
    issue_tile(tile + kTileBufs);
  }

  // ---- O (FP32 [head][dim]), maxima and denominators to shared memory
  float* so = reinterpret_cast<float*>(s.k[0]);
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    const int dim = (2 * warp + mt) * 16 + fg;
    so[(2 * cq) * kHeadDim + dim] = o[mt][0];
    so[(2 * cq + 1) * kHeadDim + dim] = o[mt][1];
    so[(2 * cq) * kHeadDim + dim + 8] = o[mt][2];
    so[(2 * cq + 1) * kHeadDim + dim + 8] = o[mt][3];
  }
  if (warp == 0 && fg == 0) {
    s.m[2 * cq] = mrun[0];
    s.m[2 * cq + 1] = mrun[1];
  }
  __syncthreads();
  if (tid < 8) {
    float l = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w)
      l += s.l[w][tid];
    s.lsum[tid] = l;
  }
  __syncthreads();
  const int d = tid;
  float acc[G];
#pragma unroll
  for (int h = 0; h < G; ++h)
    acc[h] = so[h * kHeadDim + d];
  if (used == 1) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const int head = g * G + h;
      const float gate = p.gate[size_t(r) * p.ldg + head];
      const float y = (acc[h] / s.lsum[h]) / (1 + expf(-gate));
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
      out[1] = s.lsum[h];
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
  // every span's maximum and denominator at once, then the span weights
  // exp(m_sp - max) per head (one thread per head), then the outputs
  float* mw = so + 8 * kHeadDim;  // [span][8]
  float* lw = mw + 8 * kMaxDecodeSplits;
  for (int i = tid; i < used * G; i += kThreads) {
    const int sp = i / G, h = i % G;
    const float* pp = part(sp, g * G + h);
    mw[sp * 8 + h] = __ldcg(pp);
    lw[sp * 8 + h] = __ldcg(pp + 1);
  }
  __syncthreads();
  if (tid < G) {
    float maximum = -INFINITY;
    for (int sp = 0; sp < used; ++sp)
      maximum = fmaxf(maximum, mw[sp * 8 + tid]);
    float sum = 0;
    for (int sp = 0; sp < used; ++sp) {
      const float w = expf(mw[sp * 8 + tid] - maximum);
      mw[sp * 8 + tid] = w;
      sum = fmaf(lw[sp * 8 + tid], w, sum);
    }
    s.lsum[tid] = sum;
  }
  __syncthreads();
  // the spans' values in chunks whose loads are all in flight at once,
  // accumulated in span order
  constexpr int kChunk = 32 / G;
  float value[G];
#pragma unroll
  for (int h = 0; h < G; ++h)
    value[h] = 0;
  for (int sp0 = 0; sp0 < used; sp0 += kChunk) {
    float x[kChunk][G];
#pragma unroll
    for (int j = 0; j < kChunk; ++j)
#pragma unroll
      for (int h = 0; h < G; ++h)
        x[j][h] = sp0 + j < used ? __ldcg(part(sp0 + j, g * G + h) + 2 + d)
                                 : 0.0F;
#pragma unroll
    for (int j = 0; j < kChunk; ++j)
#pragma unroll
      for (int h = 0; h < G; ++h)
        if (sp0 + j < used)
          value[h] = fmaf(x[j][h], mw[(sp0 + j) * 8 + h], value[h]);
  }
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const int head = g * G + h;
    const float gate = p.gate[size_t(r) * p.ldg + head];
    const float y = (value[h] / s.lsum[h]) / (1 + expf(-gate));
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
  if (const cudaError_t e = ensure_dynamic_smem(
          reinterpret_cast<const void*>(decode_attention_kernel<G>),
          int(sizeof(DecodeSmem))))
    return e;
  config.gridDim = dim3(p.kv_heads, spans, rows);
  config.blockDim = dim3(kThreads);
  config.dynamicSmemBytes = sizeof(DecodeSmem);
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

int decode_key_tiles(int position, int window) {
  const int first = window > 0 ? max(0, position + 1 - window) : 0;
  return (position + 1 - first + kDecodeTile - 1) / kDecodeTile;
}

int decode_spans_used(int position, int window, int max_splits,
                      int span_tiles) {
  const int tiles = decode_key_tiles(position, window);
  const int per = decode_span_tiles(tiles, max_splits, span_tiles);
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
