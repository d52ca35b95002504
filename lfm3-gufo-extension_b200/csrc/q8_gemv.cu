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
#include "q8_gemv.cuh"
#include "kernels.cuh"

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

// Source row of tile row i, or nullptr past the weights.
__device__ __forceinline__ const uint8_t* tile_source(const GemvParams& p,
                                                      int t, int i,
                                                      size_t row_bytes) {
  if (p.kind == kGemvPlain) {
    int j = 0;
#pragma unroll
    for (int q = 1; q < 4; ++q)
      if (q < p.n_out && t >= p.first_tile[q])
        j = q;
    const int row = (t - p.first_tile[j]) * kGemvRows + i;
    return row < p.o[j].rows ? p.o[j].w + size_t(row) * row_bytes : nullptr;
  }
  if (p.kind == kGemvSwiGLU) {
    const int row = t * 32 + (i & 31);
    if (row >= p.o[0].rows)
      return nullptr;
    return p.o[i < 32 ? 0 : 1].w + size_t(row) * row_bytes;
  }
  // Conv: rows 0-15 B, 16-31 C, 32-47 x of channels 16t..16t+15
  const int ch = t * 16 + (i & 15);
  if (i >= 48 || ch >= p.H)
    return nullptr;
  return p.o[0].w + (size_t(i / 16) * p.H + ch) * row_bytes;
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

__global__ void __launch_bounds__(kGemvThreads, 1)
    q8_gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  GemvSmem& s = *reinterpret_cast<GemvSmem*>(smem_raw);
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const long long units = (long long)p.tiles * p.chunks;
  const long long grid = gridDim.x;
  const long long u0 = unit_begin(blockIdx.x, units, grid);
  const long long u1 = unit_begin(blockIdx.x + 1, units, grid);
  const size_t row_bytes = size_t(p.K / 32) * 34;

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
      const uint8_t* src0 = tile_source(p, t, lane, row_bytes);
      const uint8_t* src1 = tile_source(p, t, lane + 32, row_bytes);
      const unsigned n0 = __popc(__ballot_sync(0xffffffffu, src0 != nullptr));
      const unsigned n1 = __popc(__ballot_sync(0xffffffffu, src1 != nullptr));
      if (lane == 0)
        mbar_arrive_expect_tx(&s.full[stage], (n0 + n1) * kGemvChunk);
      __syncwarp();
      uint8_t* dst = s.stage[stage];
      if (src0)
        bulk_load(dst + lane * kGemvChunk, src0 + size_t(c) * kGemvChunk,
                  kGemvChunk, &s.full[stage]);
      if (src1)
        bulk_load(dst + (lane + 32) * kGemvChunk,
                  src1 + size_t(c) * kGemvChunk, kGemvChunk, &s.full[stage]);
      if (++stage == kGemvStages) {
        stage = 0;
        phase ^= 1;
      }
    }
    return;
  }

  // ---- consumers
  grid_dependency_wait();
  const int g = lane / 4, cq = lane % 4;
  const int mtiles = p.kind == kGemvConv ? 3 : 4;
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
    const uint8_t* base = s.stage[stage] + warp * 34;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      if (m >= mtiles)
        break;
      uint32_t w[2][2];  // [row g / g + 8][codes 0-3 / 4-7]
      float d[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint8_t* row = base + (m * 16 + g + h * 8) * kGemvChunk;
        d[h] = __half2float(*reinterpret_cast<const __half*>(row));
        const uint8_t* q = row + 2 + 8 * cq;
        // Odd g reads its words in the other order, so a warp's 32 lanes
        // cover 32 banks (the row pitch is 4 words modulo 32).
        if (warp & 1) {  // codes start on a word
          const uint32_t* pw = reinterpret_cast<const uint32_t*>(q);
          const uint32_t a = pw[g & 1], b = pw[(g & 1) ^ 1];
          w[h][0] = (g & 1) ? b : a;
          w[h][1] = (g & 1) ? a : b;
        } else {  // codes start two bytes into a word
          const uint32_t* pw = reinterpret_cast<const uint32_t*>(q - 2);
          uint32_t v0, v1, v2;
          if (g & 1) {
            v1 = pw[1];
            v2 = pw[2];
            v0 = pw[0];
          } else {
            v0 = pw[0];
            v1 = pw[1];
            v2 = pw[2];
          }
          w[h][0] = __funnelshift_r(v0, v1, 16);
          w[h][1] = __funnelshift_r(v1, v2, 16);
        }
      }
      uint32_t a1[4], a2[4];
      codes_to_half2(w[0][0], a1[0], a1[2]);
      codes_to_half2(w[1][0], a1[1], a1[3]);
      codes_to_half2(w[0][1], a2[0], a2[2]);
      codes_to_half2(w[1][1], a2[1], a2[3]);
      float cc[4] = {0, 0, 0, 0};
      mma_f16(cc, a1, xh.x, xh.y);
      mma_f16(cc, a1, xl.x, xl.y);
      mma_f16(cc, a2, xh.z, xh.w);
      mma_f16(cc, a2, xl.z, xl.w);
      acc[m][0] = fmaf(d[0], cc[0], acc[m][0]);
      acc[m][1] = fmaf(d[0], cc[1], acc[m][1]);
      acc[m][2] = fmaf(d[1], cc[2], acc[m][2]);
      acc[m][3] = fmaf(d[1], cc[3], acc[m][3]);
    }
    __syncwarp();
    if (lane == 0)
      mbar_arrive(&s.empty[stage]);
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

}  // namespace

int gemv_grid(int units, int sms) { return units < sms ? units : sms; }

size_t gemv_partial_floats(int grid) { return size_t(grid) * 2 * kGemvTile; }

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
