// Q8_0 projections of up to eight FP32 rows; see q8_gemv.cuh.
//
// Layout of the work: a tile is 64 weight rows over all K columns; a unit is
// one tile's 256-column chunk (8 Q8 blocks, 272 bytes per row). The
// tiles x chunks units of a launch are dealt to the CTAs as contiguous
// ranges (stream-K), so every CTA streams the same number of weight bytes.
// A producer warp copies each unit's 64 row pieces into a ring of shared
// memory stages with bulk copies; eight consumer warps take one Q8 block
// each per unit and run it on the tensor cores:
//
//   A = the block's codes of 16 rows, decoded exactly to fp16
//   B = the input rows as two fp16 terms (hi, lo) of up to 8 tokens
//   C = sum over the block's 32 columns, FP32, then acc += d * C
//
// i.e. the reference's per-block order "sum += d * (sum of q * x)"
// (hip/ops.hip:784-809) with FP32 accumulation. Inside a block the 32
// columns are assigned to MMA k positions by a fixed permutation that the
// split-activation records follow, so every thread reads 8 contiguous codes.
// Warp partials merge through shared memory in warp order; a tile split
// between CTAs merges its parts in CTA order in whichever CTA finishes it
// last (a ticket, not a wait), so results never depend on timing.
#include "common.cuh"
#include "kernels.cuh"
#include "q8_gemv.cuh"
#include "tensor_map.hpp"

namespace lfm3 {

namespace {

struct GemvSmem {
  uint8_t stage[kGemvStages][kGemvRows * kGemvChunk];
  float red[kGemvWarps][kGemvTile];
  float tile[kGemvTile];
  uint64_t full[kGemvStages];
  uint64_t empty[kGemvStages];
  int last;
};

// Issues the tiled copies of unit (tile t, chunk c) into `dst`; returns the
// bytes they deliver (boxes past the matrix are zero-filled and still count).
__device__ __forceinline__ uint32_t load_unit(const GemvParams& p, int t,
                                              int c, uint8_t* dst,
                                              uint64_t* bar) {
  const int x1 = c * (kGemvChunk / 16);
  if (p.kind == kGemvPlain) {
    int j = 0;
#pragma unroll
    for (int q = 1; q < 4; ++q)
      if (q < p.n_out && t >= p.first_tile[q])
        j = q;
    tma_load_3d(dst, &p.maps[j], 0, x1, (t - p.first_tile[j]) * kGemvRows,
                bar);
    return kGemvRows * kGemvChunk;
  }
  if (p.kind == kGemvSwiGLU) {
    tma_load_3d(dst, &p.maps[0], 0, x1, t * 32, bar);
    tma_load_3d(dst + 32 * kGemvChunk, &p.maps[1], 0, x1, t * 32, bar);
    return kGemvRows * kGemvChunk;
  }
  // Conv: rows 0-15 B, 16-31 C, 32-47 x of channels 16t..16t+15
#pragma unroll
  for (int part = 0; part < 3; ++part)
    tma_load_3d(dst + part * 16 * kGemvChunk, &p.maps[0], 0, x1,
                part * p.H + t * 16, bar);
  return 48 * kGemvChunk;
}

__device__ __forceinline__ long long unit_begin(long long c, long long units,
                                                long long grid) {
  return c * units / grid;
}
// The CTA whose range holds unit u.
__device__ __forceinline__ int unit_owner(long long u, long long units,
                                          long long grid) {
  return int(((u + 1) * grid - 1) / units);
}

__device__ void gemv_epilogue(const GemvParams& p, const float* tile, int t,
                              int tid) {
  const int tokens = p.tokens;
  if (p.kind == kGemvPlain) {
    int j = 0;
#pragma unroll
    for (int q = 1; q < 4; ++q)
      if (q < p.n_out && t >= p.first_tile[q])
        j = q;
    const int row0 = (t - p.first_tile[j]) * kGemvRows;
    for (int e = tid; e < kGemvTile; e += kGemvWarps * 32) {
      const int i = e / kMaxBatch, tok = e % kMaxBatch;
      const int row = row0 + i;
      if (tok < tokens && row < p.o[j].rows)
        p.o[j].out[size_t(tok) * p.o[j].ld + row] = tile[e];
    }
    return;
  }
  if (p.kind == kGemvSwiGLU) {
    // 32 rows x 8 tokens
    const int i = tid / kMaxBatch, tok = tid % kMaxBatch;
    const int row = t * 32 + i;
    if (i < 32 && tok < tokens && row < p.o[0].rows) {
      const float g = tile[i * kMaxBatch + tok];
      const float u = tile[(32 + i) * kMaxBatch + tok];
      // BatchedSwiGLUActivationKernel's formula (hip/ops.hip:175-177)
      const float sig = 1.0F / (1.0F + expf(-g));
      const float h = (g * sig) * u;
      if (p.split_out)
        store_split(p.split_out, tok, p.split_width, row, h);
      if (p.o[0].out)
        p.o[0].out[size_t(tok) * p.o[0].ld + row] = h;
    }
    return;
  }
  // Conv step per (channel, token), ConvolutionStep's expressions
  // (hip/ops.hip:1135-1151): FMA chain over the window oldest first, then
  // gate by C; the history shifts by one and keeps the newest B*x.
  const int i = tid / kMaxBatch, tok = tid % kMaxBatch;
  const int ch = t * 16 + i;
  if (i < 16 && tok < tokens && ch < p.H) {
    const int L = p.L;
    const float b = tile[i * kMaxBatch + tok];
    const float c = tile[(16 + i) * kMaxBatch + tok];
    const float x = tile[(32 + i) * kMaxBatch + tok];
    float* own = p.rows->layers[tok][p.layer].conv + size_t(ch) * (L - 1);
    const float* w = p.conv_w + size_t(ch) * L;
    const float current = b * x;
    float sum = 0;
    for (int j = 0; j < L - 1; ++j)
      sum = fmaf(w[j], own[j], sum);
    sum = fmaf(w[L - 1], current, sum);
    for (int j = 0; j < L - 2; ++j)
      own[j] = own[j + 1];
    own[L - 2] = current;
    store_split(p.split_out, tok, p.split_width, ch, sum * c);
  }
}

// The block of this warp (codes of rows m * 16 + g and + 8, 8 codes per
// thread) as MMA A fragments for the chunk's two k16 halves.
template <bool kAligned, int kMTiles>
__device__ __forceinline__ void load_block(const uint8_t* base, int g, int cq,
                                           uint32_t (&a1)[kMTiles][4],
                                           uint32_t (&a2)[kMTiles][4],
                                           float (&d)[kMTiles][2]) {
  uint32_t w[kMTiles][2][2];
#pragma unroll
  for (int m = 0; m < kMTiles; ++m)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint8_t* row = base + (m * 16 + g + h * 8) * kGemvChunk;
      d[m][h] = __half2float(*reinterpret_cast<const __half*>(row));
      if (kAligned) {
        const uint32_t* pw = reinterpret_cast<const uint32_t*>(row + 2 + 8 * cq);
        w[m][h][0] = pw[0];
        w[m][h][1] = pw[1];
      } else {
        const uint32_t* pw = reinterpret_cast<const uint32_t*>(row + 8 * cq);
        const uint32_t v0 = pw[0], v1 = pw[1], v2 = pw[2];
        w[m][h][0] = __funnelshift_r(v0, v1, 16);
        w[m][h][1] = __funnelshift_r(v1, v2, 16);
      }
    }
#pragma unroll
  for (int m = 0; m < kMTiles; ++m) {
    codes_to_half2(w[m][0][0], a1[m][0], a1[m][2]);
    codes_to_half2(w[m][1][0], a1[m][1], a1[m][3]);
    codes_to_half2(w[m][0][1], a2[m][0], a2[m][2]);
    codes_to_half2(w[m][1][1], a2[m][1], a2[m][3]);
  }
}

template <bool kAligned, int kMTiles>
__device__ __forceinline__ void consume(const GemvParams& p, GemvSmem& s,
                                        long long u0, long long u1,
                                        long long units, long long grid,
                                        int tid, int warp, int lane) {
  const int g = lane / 4, cq = lane % 4;
  const uint4* x = static_cast<const uint4*>(p.x);
  const int records = p.K / 8;
  int stage = 0;
  uint32_t phase = 0;
  float acc[4][4];
  const int first_tile = int(u0 / p.chunks);
  for (long long u = u0; u < u1; ++u) {
    const int t = int(u / p.chunks), c = int(u % p.chunks);
    if (u == u0 || c == 0) {
#pragma unroll
      for (int m = 0; m < 4; ++m)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          acc[m][j] = 0;
    }
    // this warp's block of the chunk; its input terms for token g
    const int kb = c * kGemvBlocks + warp;
    uint4 xh = make_uint4(0, 0, 0, 0), xl = xh;
    if (g < p.tokens) {
      const uint4* rec = x + (size_t(g) * records + kb * 4 + cq) * 2;
      xh = __ldg(rec);
      xl = __ldg(rec + 1);
    }
    if (!mbar_wait(&s.full[stage], phase, kErrGemvFullWait))
      return;
    {
      uint32_t a1[kMTiles][4], a2[kMTiles][4];
      float d[kMTiles][2];
      load_block<kAligned, kMTiles>(s.stage[stage] + warp * 34, g, cq, a1, a2,
                                    d);
      __syncwarp();
      if (lane == 0)
        mbar_arrive(&s.empty[stage]);
#pragma unroll
      for (int m = 0; m < kMTiles; ++m) {
        float cc[4] = {0, 0, 0, 0};
        mma_f16(cc, a1[m], xh.x, xh.y);
        mma_f16(cc, a1[m], xl.x, xl.y);
        mma_f16(cc, a2[m], xh.z, xh.w);
        mma_f16(cc, a2[m], xl.z, xl.w);
        acc[m][0] = fmaf(d[m][0], cc[0], acc[m][0]);
        acc[m][1] = fmaf(d[m][0], cc[1], acc[m][1]);
        acc[m][2] = fmaf(d[m][1], cc[2], acc[m][2]);
        acc[m][3] = fmaf(d[m][1], cc[3], acc[m][3]);
      }
    }
    if (++stage == kGemvStages) {
      stage = 0;
      phase ^= 1;
    }
    // ---- end of this CTA's part of tile t
    if (c + 1 < p.chunks && u + 1 < u1)
      continue;
    float* red = s.red[warp];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int r = m * 16 + g;
      red[r * kMaxBatch + 2 * cq] = acc[m][0];
      red[r * kMaxBatch + 2 * cq + 1] = acc[m][1];
      red[(r + 8) * kMaxBatch + 2 * cq] = acc[m][2];
      red[(r + 8) * kMaxBatch + 2 * cq + 1] = acc[m][3];
    }
    named_barrier(1, kGemvWarps * 32);
    for (int e = tid; e < kGemvTile; e += kGemvWarps * 32) {
      float v = s.red[0][e];
#pragma unroll
      for (int q = 1; q < kGemvWarps; ++q)
        v += s.red[q][e];
      s.tile[e] = v;
    }
    const long long tu0 = (long long)t * p.chunks;
    const int c_first = unit_owner(tu0, units, grid);
    const int c_last = unit_owner(tu0 + p.chunks - 1, units, grid);
    if (c_first != c_last) {
      // part of a tile shared with other CTAs: publish, take a ticket
      const int slot = t == first_tile ? 0 : 1;
      float* mine = p.partials + (size_t(blockIdx.x) * 2 + slot) * kGemvTile;
      for (int e = tid; e < kGemvTile; e += kGemvWarps * 32)
        mine[e] = s.tile[e];
      __threadfence();
      named_barrier(1, kGemvWarps * 32);
      if (tid == 0) {
        const unsigned parts = unsigned(c_last - c_first + 1);
        const unsigned old = atomicAdd(&p.tickets[t], 1u);
        s.last = old == parts - 1;
        if (s.last)
          p.tickets[t] = 0;
      }
      named_barrier(1, kGemvWarps * 32);
      if (!s.last)
        continue;
      __threadfence();
      for (int e = tid; e < kGemvTile; e += kGemvWarps * 32) {
        float v = 0;
        for (int q = c_first; q <= c_last; ++q) {
          const int q_first = int(unit_begin(q, units, grid) / p.chunks);
          const float* part =
              p.partials + (size_t(q) * 2 + (t == q_first ? 0 : 1)) * kGemvTile;
          const float pv = __ldcg(part + e);
          v = q == c_first ? pv : v + pv;
        }
        s.tile[e] = v;
      }
    }
    named_barrier(1, kGemvWarps * 32);
    gemv_epilogue(p, s.tile, t, tid);
    named_barrier(1, kGemvWarps * 32);
  }
}


__global__ void __launch_bounds__(kGemvThreads, 2)
    q8_gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  GemvSmem& s = *reinterpret_cast<GemvSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const long long units = (long long)p.tiles * p.chunks;
  const long long grid = gridDim.x;
  const long long u0 = unit_begin(blockIdx.x, units, grid);
  const long long u1 = unit_begin(blockIdx.x + 1, units, grid);
  if (tid == 0) {
    for (int i = 0; i < kGemvStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], kGemvWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  allow_dependents();

  if (warp == kGemvWarps) {
    // ---- producer: weights only, so it may run ahead of the previous
    // kernel in the stream
    int stage = 0;
    uint32_t phase = 0;
    for (long long u = u0; u < u1; ++u) {
      const int t = int(u / p.chunks), c = int(u % p.chunks);
      if (!mbar_wait(&s.empty[stage], phase ^ 1, kErrGemvEmptyWait))
        return;
      if (lane == 0) {
        const uint32_t bytes =
            p.kind == kGemvConv ? 48 * kGemvChunk : kGemvRows * kGemvChunk;
        mbar_arrive_expect_tx(&s.full[stage], bytes);
        load_unit(p, t, c, s.stage[stage], &s.full[stage]);
      }
      __syncwarp();
      if (++stage == kGemvStages) {
        stage = 0;
        phase ^= 1;
      }
    }
    return;
  }

  // ---- consumers
  grid_dependency_wait();
  // Odd warps' blocks start on a word boundary, even warps' two bytes past
  // one; each variant is straight-line code over the tile's m-tiles.
  if (warp & 1) {
    if (p.kind == kGemvConv)
      consume<true, 3>(p, s, u0, u1, units, grid, tid, warp, lane);
    else
      consume<true, 4>(p, s, u0, u1, units, grid, tid, warp, lane);
  } else {
    if (p.kind == kGemvConv)
      consume<false, 3>(p, s, u0, u1, units, grid, tid, warp, lane);
    else
      consume<false, 4>(p, s, u0, u1, units, grid, tid, warp, lane);
  }
}

}  // namespace

int gemv_grid(int units, int sms) { return units < sms ? units : sms; }

size_t gemv_partial_floats(int grid) { return size_t(grid) * 2 * kGemvTile; }

cudaError_t fill_gemv_maps(GemvParams& p) {
  const size_t row_bytes = size_t(p.K / 32) * 34;
  const int outputs = p.kind == kGemvPlain ? p.n_out : p.kind == kGemvSwiGLU ? 2 : 1;
  for (int j = 0; j < outputs; ++j) {
    const cudaError_t e =
        encode_row_map(&p.maps[j], p.o[j].w, row_bytes, p.o[j].rows,
                       kGemvChunk, gemv_box_rows(p.kind));
    if (e != cudaSuccess)
      return e;
  }
  return cudaSuccess;
}

cudaError_t launch_q8_gemv(const GemvParams& p, int grid, cudaStream_t stream,
                           bool pdl) {
  static bool configured = false;
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(
        q8_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
        int(sizeof(GemvSmem)));
    if (e != cudaSuccess)
      return e;
    configured = true;
  }
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
