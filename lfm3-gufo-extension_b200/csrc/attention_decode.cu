// Decode attention for every row of a round in one launch.
//
// Grid (kv_heads, splits, rows): a CTA owns one KV group of one row and a
// span of that row's keys, so ragged depths need no per-row launches. Every
// CTA normalises and rotates its group's query heads itself (cheap), and the
// CTA whose span ends at the row's position also stores the new K/V row in
// the ring. Keys stream through shared memory in tiles of 64, three tiles in
// flight; warp w copies and consumes keys 16 w .. 16 w + 15 of every tile
// and keeps its own online softmax (FP32 scores, probabilities and
// accumulators: the decode precision of hip/ops.hip:1562-1691), so warps
// never wait for one another inside the key loop; the four warps' states
// merge once at the end. Both products run on the tensor cores (mma.sync
// m16n8k16, FP32 accumulation) with the FP32 operands split in two fp16
// terms, x = hi + lo (22 significant bits): S^T = K (Q_hi + Q_lo)^T with the
// warp's 16 keys as M and the group's heads (padded to 8) as N, then
// O^T += V^T (P_hi + P_lo)^T with the 128 dimensions as M, the probability
// fragments transposed in registers (movmatrix); K and V are the cache's
// fp16 values, exactly. With several spans, each CTA writes its maximum,
// denominator and unnormalised output, and whichever CTA of the group
// finishes last (a ticket, not a wait) merges them in span order and applies
// the gate (hip/ops.hip:1710-1728).
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

// Three key tiles in flight: K and V of tile t in buffer t % 3.
constexpr int kTileBufs = 3;
constexpr int kWarpKeys = kDecodeTile / kWarps;  // keys of a tile per warp
static_assert(kWarpKeys == 16, "one m16 key block per warp and tile");
struct DecodeSmem {
  alignas(16) __half k[kTileBufs][kDecodeTile * kHeadDim];  // [key][dim]
  alignas(16) __half v[kTileBufs][kDecodeTile * kHeadDim];  // [key][dim]
  alignas(16) __half qh[8 * kHeadDim], ql[8 * kHeadDim];      // [head][dim]
  float wm[kWarps][8], wl[kWarps][8];  // each warp's maxima, denominators
  float ws[kWarps][8];                 // each warp's merge weight
  float m[8], lsum[8];
  alignas(16) __half newk[kHeadDim], newv[kHeadDim];  // the row at `position`
  int last;
};
// After the key loop the K buffers hold the warps' outputs
// ([warp][head][dim], FP32) and then the span merge weights.
static_assert(sizeof(float) *
                      (kWarps * 8 * kHeadDim + 2 * 8 * kMaxDecodeSplits) <=
                  sizeof(__half) * kTileBufs * kDecodeTile * kHeadDim,
              "output staging fits the K buffers");

// 16 bytes global -> shared, zero-filled when !valid (cp.async, L1
// bypassed), under an L2 cache policy (the keys and values of a layer are
// read once per round)
__device__ __forceinline__ void cp_async16(void* dst, const void* src,
                                           bool valid, uint64_t policy) {
  asm volatile(
      "cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(valid ? 16 : 0), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// every group but the newest kTileBufs - 1 has landed (this thread's copies)
__device__ __forceinline__ void cp_async_wait_oldest() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kTileBufs - 1) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// The transpose of an 8 x 8 fp16 matrix held one element pair per thread
// (the mma fragment layout: thread t has row t / 4, columns 2 (t % 4) and
// 2 (t % 4) + 1), within the warp.
__device__ __forceinline__ uint32_t transpose8x8(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;"
               : "=r"(d)
               : "r"(a));
  return d;
}
__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
  return uint32_t(__half_as_ushort(lo)) |
         (uint32_t(__half_as_ushort(hi)) << 16);
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

// Two CTAs per SM (96 KB of key tiles each): a round's spans run in about
// one wave.
template <int G>
__global__ void __launch_bounds__(kThreads, 2)
    decode_attention_kernel(const __grid_constant__ DecodeAttentionParams p) {
  extern __shared__ __align__(128) uint8_t decode_smem_raw[];
  DecodeSmem& s = *reinterpret_cast<DecodeSmem*>(decode_smem_raw);
  const int g = blockIdx.x, split = blockIdx.y, r = blockIdx.z;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  // ---- before the dependency wait: the row table (written before the
  // round), the launch's constants and, with settled rings, the first key
  // tiles
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

  // ---- this warp's 16 keys of a tile (K and V rows as 16-byte pieces)
  // copied into buffer (tile % kTileBufs); one cp.async group per tile
  // (empty past the span)
  const int wkey = warp * kWarpKeys;  // the warp's first key in a tile
  const uint64_t policy = l2_evict_first_policy();
  const auto issue_tile = [&](int tile) {
    const int base = begin + tile * kDecodeTile + wkey;
    if (base < end) {
      const int n = min(kWarpKeys, end - base);
      const int slot0 = base % capacity;  // ring slot of key `base`
      __half* sk = s.k[tile % kTileBufs];
      __half* sv = s.v[tile % kTileBufs];
#pragma unroll
      for (int j = 0; j < kWarpKeys * 16 / 32; ++j) {
        const int c = lane + j * 32, key = c / 16, piece = c % 16;
        const int kk = min(key, n - 1);
        const int t = base + kk;
        const __half *ks = state.k, *vs = state.v;
        int slot = slot0 + kk;
        if (slot >= capacity)
          slot = capacity >= kWarpKeys ? slot - capacity : slot % capacity;
        size_t row = size_t(slot) * stride;
        if (op && t >= position) {
          ks = p.chunk_k;
          vs = p.chunk_v;
          row = size_t(t - position) * stride;
        }
        row += size_t(g) * kHeadDim;
        cp_async16(&sk[at128(wkey + key, piece)],
                   reinterpret_cast<const uint4*>(ks + row) + piece, key < n,
                   policy);
        cp_async16(&sv[at128(wkey + key, piece)],
                   reinterpret_cast<const uint4*>(vs + row) + piece, key < n,
                   policy);
      }
    }
    cp_async_commit();
  };
  // with settled rings the first tiles are copied while the previous
  // kernel finishes (the row at `position` is patched in below)
  const bool early = !op && p.ring_settled;
  if (early)
#pragma unroll
    for (int i = 0; i < kTileBufs; ++i)
      issue_tile(i);
  grid_dependency_wait();
  allow_dependents();
  if (!early)
#pragma unroll
    for (int i = 0; i < kTileBufs; ++i)
      issue_tile(i);

  // ---- query heads of this group (normalised, rotated), as hi + lo fp16
  // terms; heads G..7 are zero. The new key and value of the row are read
  // together with the queries.
  float nk0[2] = {0, 0}, nk1[2] = {0, 0}, nv[4] = {0, 0, 0, 0};
  const bool new_row = stores_row && warp == 0;
  float gate[G];  // the group's gates, used once the span is done
#pragma unroll
  for (int h = 0; h < G; ++h)
    gate[h] = p.gate[size_t(r) * p.ldg + g * G + h];
  if (new_row) {
    const float* kx = p.k + size_t(r) * p.ldk + size_t(g) * kHeadDim;
    const float* vx = p.v + size_t(r) * p.ldk + size_t(g) * kHeadDim;
    nk0[0] = kx[lane], nk0[1] = kx[lane + 32];
    nk1[0] = kx[lane + 64], nk1[1] = kx[lane + 96];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      nv[j] = vx[lane + 32 * j];
  }
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
  if (new_row) {
    norm_rope(nk0, nk1, kn, rot, p.eps);
    const size_t slot = size_t(position % capacity) * stride +
                        size_t(g) * kHeadDim;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int i = lane + 32 * j;
      const __half k0 = __float2half_rn(nk0[j]), k1 = __float2half_rn(nk1[j]);
      const __half v0 = __float2half_rn(nv[j]), v1 = __float2half_rn(nv[j + 2]);
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
  __syncthreads();

  // fragment coordinates: row fg (and fg + 8), column pair 2 cq, 2 cq + 1
  const int fg = lane / 4, cq = lane % 4;
  // ldmatrix lane roles: matrix mj = lane / 8 takes its row from lane mrow
  const int mj = lane / 8, mrow = lane % 8;
  // the queries as the B operand of S^T = K Q^T, for the whole span
  uint32_t qbh[kHeadDim / 16][2], qbl[kHeadDim / 16][2];
#pragma unroll
  for (int ks = 0; ks < kHeadDim / 16; ++ks) {
    ldsm_x2(qbh[ks], &s.qh[at128(mrow, 2 * ks + (mj & 1))]);
    ldsm_x2(qbl[ks], &s.ql[at128(mrow, 2 * ks + (mj & 1))]);
  }
  // this warp's running maxima and denominators of heads 2 cq, 2 cq + 1
  // (every lane holds the same values) and its O^T fragments: dimension
  // tile mt, rows 16 mt + fg (+ 8), heads 2 cq, 2 cq + 1
  float mrun[2] = {-INFINITY, -INFINITY}, lrun[2] = {0, 0};
  float o[kHeadDim / 16][4];
#pragma unroll
  for (int mt = 0; mt < kHeadDim / 16; ++mt)
    o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0;

  for (int tile = 0, base = begin; base < end; ++tile, base += kDecodeTile) {
    const int n = min(kDecodeTile, end - base) - wkey;  // the warp's keys
    __half* const tk = s.k[tile % kTileBufs];
    __half* const tv = s.v[tile % kTileBufs];
    cp_async_wait_oldest();  // this tile's group (the next ones may fly)
    __syncwarp();
    if (n > 0) {
      if (stores_row && position >= base + wkey &&
          position < base + wkey + n) {
        // the ring slot may have been copied before this CTA wrote it
        const int key = position - base;
        if (lane < 16)
          *reinterpret_cast<uint4*>(&tk[at128(key, lane)]) =
              *reinterpret_cast<const uint4*>(&s.newk[lane * 8]);
        else
          *reinterpret_cast<uint4*>(&tv[at128(key, lane - 16)]) =
              *reinterpret_cast<const uint4*>(&s.newv[(lane - 16) * 8]);
        __syncwarp();
      }
      // ---- S^T = K Q^T over the warp's 16 keys, two accumulation chains
      float sa[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
      float sb[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
      const int krow = wkey + (mj & 1) * 8 + mrow;
#pragma unroll
      for (int ks = 0; ks < kHeadDim / 16; ++ks) {
        uint32_t a[4];
        ldsm_x4(a, &tk[at128(krow, 2 * ks + (mj >> 1))]);
        mma_f16(sa[ks & 1], a, qbh[ks][0], qbh[ks][1]);
        mma_f16(sb[ks & 1], a, qbl[ks][0], qbl[ks][1]);
      }
      // this thread: keys fg and fg + 8 of the warp's block, heads 2 cq and
      // 2 cq + 1
      float sc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        sc[i] = ((sa[0][i] + sa[1][i]) + (sb[0][i] + sb[1][i])) * kScoreScale;
      if (fg >= n)
        sc[0] = sc[1] = -INFINITY;
      if (fg + 8 >= n)
        sc[2] = sc[3] = -INFINITY;
      float t0 = fmaxf(sc[0], sc[2]), t1 = fmaxf(sc[1], sc[3]);
#pragma unroll
      for (int x = 4; x < 32; x <<= 1) {
        t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, x));
        t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, x));
      }
      // ---- online softmax over the warp's keys (the block's first key is
      // live, so the maxima are finite)
      const float top[2] = {fmaxf(mrun[0], t0), fmaxf(mrun[1], t1)};
      const float alpha[2] = {expf(mrun[0] - top[0]),  // 0 at the first block
                              expf(mrun[1] - top[1])};
      mrun[0] = top[0];
      mrun[1] = top[1];
      const float pr[4] = {expf(sc[0] - top[0]), expf(sc[1] - top[1]),
                           expf(sc[2] - top[0]), expf(sc[3] - top[1])};
      float q0 = pr[0] + pr[2], q1 = pr[1] + pr[3];
#pragma unroll
      for (int x = 4; x < 32; x <<= 1) {
        q0 += __shfl_xor_sync(0xffffffffu, q0, x);
        q1 += __shfl_xor_sync(0xffffffffu, q1, x);
      }
      lrun[0] = lrun[0] * alpha[0] + q0;
      lrun[1] = lrun[1] * alpha[1] + q1;
      // P^T as the B operand: the 16 x 8 (key, head) fragments transposed
      const SplitPair p0 = split_value(pr[0]), p1 = split_value(pr[1]);
      const SplitPair p2 = split_value(pr[2]), p3 = split_value(pr[3]);
      const uint32_t bh0 = transpose8x8(pack_half2(p0.hi, p1.hi));
      const uint32_t bh1 = transpose8x8(pack_half2(p2.hi, p3.hi));
      const uint32_t bl0 = transpose8x8(pack_half2(p0.lo, p1.lo));
      const uint32_t bl1 = transpose8x8(pack_half2(p2.lo, p3.lo));
      // ---- O^T += V^T P^T over all 128 dimensions
      const int vrow = wkey + (mj >> 1) * 8 + mrow;
#pragma unroll
      for (int mt = 0; mt < kHeadDim / 16; ++mt) {
        o[mt][0] *= alpha[0];
        o[mt][1] *= alpha[1];
        o[mt][2] *= alpha[0];
        o[mt][3] *= alpha[1];
        uint32_t a[4];
        ldsm_x4_trans(a, &tv[at128(vrow, 2 * mt + (mj & 1))]);
        mma_f16(o[mt], a, bh0, bh1);
        mma_f16(o[mt], a, bl0, bl1);
      }
    }
    __syncwarp();  // the warp's rows of this buffer are free
    issue_tile(tile + kTileBufs);
  }

  // ---- the warps' states merged: O (FP32 [warp][head][dim]), maxima and
  // denominators through shared memory
  cp_async_wait_all();
  __syncthreads();  // every warp is done with the key buffers
  float* wo = reinterpret_cast<float*>(s.k[0]);
#pragma unroll
  for (int mt = 0; mt < kHeadDim / 16; ++mt) {
    const int dim = mt * 16 + fg;
    float* w0 = wo + (warp * 8 + 2 * cq) * kHeadDim;
    float* w1 = w0 + kHeadDim;
    w0[dim] = o[mt][0];
    w1[dim] = o[mt][1];
    w0[dim + 8] = o[mt][2];
    w1[dim + 8] = o[mt][3];
  }
  if (fg == 0) {
    s.wm[warp][2 * cq] = mrun[0];
    s.wm[warp][2 * cq + 1] = mrun[1];
    s.wl[warp][2 * cq] = lrun[0];
    s.wl[warp][2 * cq + 1] = lrun[1];
  }
  __syncthreads();
  if (tid < 8) {
    float top = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w)
      top = fmaxf(top, s.wm[w][tid]);
    float l = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      // a warp without live keys has maximum -inf and weight 0
      const float f = s.wm[w][tid] == -INFINITY ? 0.0F : expf(s.wm[w][tid] - top);
      s.ws[w][tid] = f;
      l = fmaf(s.wl[w][tid], f, l);
    }
    s.m[tid] = top;
    s.lsum[tid] = l;
  }
  __syncthreads();
  const int d = tid;
  float acc[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float a = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w)
      a = fmaf(wo[(w * 8 + h) * kHeadDim + d], s.ws[w][h], a);
    acc[h] = a;
  }
  if (used == 1) {
#pragma unroll
    for (int h = 0; h < G; ++h) {
      const int head = g * G + h;
      const float y = (acc[h] / s.lsum[h]) / (1 + expf(-gate[h]));
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
  float* mw = wo + kWarps * 8 * kHeadDim;  // [span][8]
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
    const float y = (value[h] / s.lsum[h]) / (1 + expf(-gate[h]));
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
